/*
 * CPU oracle: plain-C restatement of torch2vk's GGUF block quantizers and
 * block decoders (Q8_0, Q4_K, Q6_K).
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (torch2vk_b200/) links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py use it, as the checker.
 *
 * Parity anchors (paths inside the torch2vk project):
 *   quantizers  src/torch2vk/quantize/vulkan.py:91-185   (Q8_0)
 *               src/torch2vk/quantize/vulkan.py:188-419  (Q4_K)
 *               src/torch2vk/quantize/vulkan.py:422-637  (Q6_K)
 *   decoders    src/models/quantized_qwen3/shaders/embedding_q4_k_f32.py:96-110 (Q4_K value)
 *               src/models/quantized_qwen3/shaders/linear_nobias_q6_k_matvec_f32.py:116-156 (Q6_K)
 *               src/models/quantized_qwen3/shaders/linear_nobias_q8_0_matvec_f32.py:84-95 (Q8_0)
 *
 * Pinning: the block layouts and decode arithmetic are pinned bit-exactly
 * against gguf-py 0.19.0 (llama.cpp's published numpy dequantizers) and the
 * reference's own GGUF reader (tests/test_oracle_pins.py).  The Q4_K / Q6_K
 * scale *search* runs only as a Vulkan shader in the reference, so its
 * restatement here is "parity unpinned" beyond the layout pin: no runnable
 * instance of the reference quantizer exists on this machine.
 *
 * Arithmetic contract (the shader's implementation-defined points, fixed here):
 *   - every float op is IEEE binary32, evaluated in source order, with no
 *     FMA contraction (the Makefile passes -ffp-contract=off);
 *   - GLSL round() in the Q6_K path is taken as round-half-away-from-zero
 *     (roundf), the choice the survey of the reference recommends;
 *   - packHalf2x16 is round-to-nearest-even (IEEE), as in the shader spec.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- fp16 --- */

static uint16_t f32_to_f16_bits(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    uint32_t sign = (bits >> 16) & 0x8000u;
    uint32_t exponent = (bits >> 23) & 0xffu;
    uint32_t mantissa = bits & 0x7fffffu;
    if (exponent == 0xffu) {
        return (uint16_t)(sign | 0x7c00u | (mantissa ? 0x200u : 0u));
    }
    int32_t half_exp = (int32_t)exponent - 127 + 15;
    if (half_exp >= 31) {
        return (uint16_t)(sign | 0x7c00u);
    }
    if (half_exp <= 0) {
        if (half_exp < -10) {
            return (uint16_t)sign;
        }
        uint32_t full = mantissa | 0x800000u;
        uint32_t shift = (uint32_t)(14 - half_exp);
        uint32_t half_mant = full >> shift;
        uint32_t rem = full & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (half_mant & 1u))) {
            half_mant += 1u;
        }
        return (uint16_t)(sign | half_mant);
    }
    uint32_t half_mant = mantissa >> 13;
    uint32_t rem = mantissa & 0x1fffu;
    uint32_t out = sign | ((uint32_t)half_exp << 10) | half_mant;
    if (rem > 0x1000u || (rem == 0x1000u && (half_mant & 1u))) {
        out += 1u; /* carries into the exponent correctly, incl. overflow to inf */
    }
    return (uint16_t)out;
}

static float f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exponent = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t mantissa = (uint32_t)h & 0x3ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            int32_t e = -1;
            do {
                e++;
                mantissa <<= 1;
            } while ((mantissa & 0x400u) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mantissa & 0x3ffu) << 13);
        }
    } else if (exponent == 0x1fu) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent - 15 + 127) << 23) | (mantissa << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

static float f16_round_trip(float value) { return f16_bits_to_f32(f32_to_f16_bits(value)); }

uint16_t t2c_oracle_f32_to_f16(float value) { return f32_to_f16_bits(value); }
float t2c_oracle_f16_to_f32(uint16_t bits) { return f16_bits_to_f32(bits); }

static float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }
static int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* ---------------------------------------------------------------- Q8_0 --- */
/* quantize/vulkan.py:143-148 round_away */
static float round_away(float value) {
    float absolute = fabsf(value);
    float floored = floorf(absolute);
    float rounded = floored + floorf(2.0f * (absolute - floored));
    float sgn = value > 0.0f ? 1.0f : (value < 0.0f ? -1.0f : 0.0f);
    return sgn * rounded;
}

/* quantize/vulkan.py:150-184: one 32-value block -> 34 bytes */
static void q8_0_block(const float *x, uint8_t *out) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) {
        amax = fmaxf(amax, fabsf(x[i]));
    }
    float block_scale = amax / 127.0f;
    float inv_scale = block_scale == 0.0f ? 0.0f : 1.0f / block_scale;
    uint16_t dh = f32_to_f16_bits(block_scale);
    out[0] = (uint8_t)(dh & 0xffu);
    out[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 32; ++i) {
        int32_t q = (int32_t)round_away(x[i] * inv_scale);
        q = clampi(q, -128, 127);
        out[2 + i] = (uint8_t)(q & 255);
    }
}

int t2c_oracle_quantize_q8_0(const float *x, int64_t rows, int64_t k, uint8_t *out) {
    if (rows < 0 || k < 0 || (k % 32) != 0) return -1;
    int64_t nb = k / 32;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            q8_0_block(x + r * k + b * 32, out + (r * nb + b) * 34);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- Q4_K --- */
/* quantize/vulkan.py:241-243 */
static uint32_t rounded_code(float value, uint32_t max_code) {
    return (uint32_t)clampf(floorf(value + 0.5f), 0.0f, (float)max_code);
}

/* quantize/vulkan.py:245-261 */
static float weighted_quant_error(const float *v, float scale, float minimum, float inv_scale) {
    float error = 0.0f;
    float sum_x2 = 0.0f;
    for (int i = 0; i < 32; ++i) sum_x2 += v[i] * v[i];
    float av_x = sqrtf(sum_x2 / 32.0f);
    for (int i = 0; i < 32; ++i) {
        float weight = av_x + fabsf(v[i]);
        float level = (float)rounded_code(inv_scale * (v[i] - minimum), 15u);
        float diff = scale * level + minimum - v[i];
        error += weight * diff * diff;
    }
    return error;
}

/* quantize/vulkan.py:263-329 */
static float choose_subblock_scale(const float *v, float *min_offset) {
    float min_value = v[0];
    float max_value = v[0];
    float sum_x2 = 0.0f;
    for (int i = 0; i < 32; ++i) {
        min_value = fminf(min_value, v[i]);
        max_value = fmaxf(max_value, v[i]);
        sum_x2 += v[i] * v[i];
    }
    if (min_value > 0.0f) min_value = 0.0f;
    if (max_value == min_value) {
        *min_offset = -min_value;
        return 0.0f;
    }
    float av_x = sqrtf(sum_x2 / 32.0f);
    float sum_w = 0.0f;
    float sum_x = 0.0f;
    for (int i = 0; i < 32; ++i) {
        float weight = av_x + fabsf(v[i]);
        sum_w += weight;
        sum_x += weight * v[i];
    }
    float inv_scale = 15.0f / (max_value - min_value);
    float best_scale = 1.0f / inv_scale;
    float best_min = min_value;
    float best_error = weighted_quant_error(v, best_scale, best_min, inv_scale);
    for (uint32_t step = 0; step <= 20u; ++step) {
        inv_scale = (14.0f + 0.1f * (float)step) / (max_value - min_value);
        float sum_l = 0.0f, sum_l2 = 0.0f, sum_xl = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float weight = av_x + fabsf(v[i]);
            float level = (float)rounded_code(inv_scale * (v[i] - min_value), 15u);
            sum_l += weight * level;
            sum_l2 += weight * level * level;
            sum_xl += weight * level * v[i];
        }
        float determinant = sum_w * sum_l2 - sum_l * sum_l;
        if (determinant > 0.0f) {
            float candidate_scale = (sum_w * sum_xl - sum_x * sum_l) / determinant;
            float candidate_min = (sum_l2 * sum_x - sum_l * sum_xl) / determinant;
            if (candidate_min > 0.0f) {
                candidate_min = 0.0f;
                candidate_scale = sum_l2 > 0.0f ? sum_xl / sum_l2 : 0.0f;
            }
            float candidate_error = weighted_quant_error(v, candidate_scale, candidate_min, inv_scale);
            if (candidate_error < best_error) {
                best_error = candidate_error;
                best_scale = candidate_scale;
                best_min = candidate_min;
            }
        }
    }
    *min_offset = fmaxf(0.0f, -best_min);
    return fmaxf(0.0f, best_scale);
}

/* quantize/vulkan.py:352-418: one 256-value super-block -> 144 bytes */
static void q4_k_block(const float *v, uint8_t *out) {
    float sub_scales[8], sub_mins[8];
    uint32_t scale_codes[8], min_codes[8];
    uint32_t quants[256];
    for (int j = 0; j < 8; ++j) {
        float min_offset = 0.0f;
        sub_scales[j] = choose_subblock_scale(v + 32 * j, &min_offset);
        sub_mins[j] = min_offset;
    }
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        max_scale = fmaxf(max_scale, sub_scales[j]);
        max_min = fmaxf(max_min, sub_mins[j]);
    }
    float d_scale = max_scale > 0.0f ? max_scale / 63.0f : 0.0f;
    float d_min = max_min > 0.0f ? max_min / 63.0f : 0.0f;
    float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
    float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    for (int j = 0; j < 8; ++j) {
        scale_codes[j] = rounded_code(sub_scales[j] * inv_scale, 63u);
        min_codes[j] = rounded_code(sub_mins[j] * inv_min, 63u);
    }
    d_scale = f16_round_trip(d_scale);
    d_min = f16_round_trip(d_min);
    for (int i = 0; i < 256; ++i) {
        int sb = i >> 5;
        float scale = d_scale * (float)scale_codes[sb];
        float minimum = d_min * (float)min_codes[sb];
        uint32_t q = 0u;
        if (scale > 0.0f) q = rounded_code((v[i] + minimum) / scale, 15u);
        quants[i] = q;
    }
    uint16_t dh = f32_to_f16_bits(d_scale);
    uint16_t mh = f32_to_f16_bits(d_min);
    out[0] = (uint8_t)(dh & 0xffu);
    out[1] = (uint8_t)(dh >> 8);
    out[2] = (uint8_t)(mh & 0xffu);
    out[3] = (uint8_t)(mh >> 8);
    /* metadata_byte, quantize/vulkan.py:331-342 */
    for (int i = 0; i < 4; ++i) {
        out[4 + i] = (uint8_t)((scale_codes[i] & 63u) | ((scale_codes[i + 4] & 48u) << 2));
        out[8 + i] = (uint8_t)((min_codes[i] & 63u) | ((min_codes[i + 4] & 48u) << 2));
        out[12 + i] = (uint8_t)((scale_codes[i + 4] & 15u) | ((min_codes[i + 4] & 15u) << 4));
    }
    /* q_byte, quantize/vulkan.py:344-350 */
    for (int b = 0; b < 128; ++b) {
        int group = b >> 5;
        int local = b & 31;
        uint32_t lo = quants[group * 64 + local] & 15u;
        uint32_t hi = quants[group * 64 + 32 + local] & 15u;
        out[16 + b] = (uint8_t)(lo | (hi << 4));
    }
}

int t2c_oracle_quantize_q4_k(const float *x, int64_t rows, int64_t k, uint8_t *out) {
    if (rows < 0 || k < 0 || (k % 256) != 0) return -1;
    int64_t nb = k / 256;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            q4_k_block(x + r * k + b * 256, out + (r * nb + b) * 144);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- Q6_K --- */
/* quantize/vulkan.py:479-481 nearest_int = int(round(value)); round() taken as half-away */
static int32_t nearest_int(float value) { return (int32_t)roundf(value); }

/* quantize/vulkan.py:483-540 */
static float make_qx_quants16(const float *v, int32_t *levels) {
    float max_value = 0.0f, max_abs = 0.0f;
    for (int i = 0; i < 16; ++i) {
        float a = fabsf(v[i]);
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
        int32_t level = clampi(nearest_int(inv_scale * v[i]), -32, 31);
        levels[i] = level + 32;
        float weight = v[i] * v[i];
        sum_lx += weight * v[i] * (float)level;
        sum_l2 += weight * (float)(level * level);
    }
    float scale = sum_l2 > 0.0f ? sum_lx / sum_l2 : 0.0f;
    float best = scale * sum_lx;
    for (int step = -9; step <= 9; ++step) {
        if (step == 0) continue;
        inv_scale = -(32.0f + 0.1f * (float)step) / max_value;
        sum_lx = 0.0f;
        sum_l2 = 0.0f;
        for (int i = 0; i < 16; ++i) {
            int32_t level = clampi(nearest_int(inv_scale * v[i]), -32, 31);
            float weight = v[i] * v[i];
            sum_lx += weight * v[i] * (float)level;
            sum_l2 += weight * (float)(level * level);
        }
        if (sum_l2 > 0.0f && sum_lx * sum_lx > best * sum_l2) {
            for (int i = 0; i < 16; ++i) {
                levels[i] = clampi(nearest_int(inv_scale * v[i]), -32, 31) + 32;
            }
            scale = sum_lx / sum_l2;
            best = scale * sum_lx;
        }
    }
    return scale;
}

/* quantize/vulkan.py:566-636: one 256-value block -> 210 bytes */
static void q6_k_block(const float *v, uint8_t *out) {
    int32_t levels[256];
    float block_scales[16];
    int32_t scale_codes[16];
    for (int g = 0; g < 16; ++g) block_scales[g] = make_qx_quants16(v + 16 * g, levels + 16 * g);
    float max_scale = 0.0f, max_abs_scale = 0.0f;
    for (int g = 0; g < 16; ++g) {
        float a = fabsf(block_scales[g]);
        if (a > max_abs_scale) {
            max_abs_scale = a;
            max_scale = block_scales[g];
        }
    }
    float d_scale;
    if (max_abs_scale < 1.0e-12f) {
        d_scale = 0.0f;
        for (int g = 0; g < 16; ++g) scale_codes[g] = 0;
    } else {
        float inv_scale = -128.0f / max_scale;
        d_scale = f16_round_trip(1.0f / inv_scale);
        for (int g = 0; g < 16; ++g) {
            scale_codes[g] = clampi(nearest_int(inv_scale * block_scales[g]), -128, 127);
        }
    }
    for (int g = 0; g < 16; ++g) {
        float d = d_scale * (float)scale_codes[g];
        if (d != 0.0f) {
            for (int i = 0; i < 16; ++i) {
                levels[16 * g + i] = clampi(nearest_int(v[16 * g + i] / d), -32, 31) + 32;
            }
        }
    }
    /* ql_byte / qh_byte, quantize/vulkan.py:542-564 */
    for (int b = 0; b < 128; ++b) {
        int section = b >> 6;
        int local = b & 31;
        int base = section * 128;
        uint32_t value;
        if ((b & 32) == 0) {
            value = ((uint32_t)levels[base + local] & 15u) | (((uint32_t)levels[base + local + 64] & 15u) << 4);
        } else {
            value = ((uint32_t)levels[base + local + 32] & 15u) | (((uint32_t)levels[base + local + 96] & 15u) << 4);
        }
        out[b] = (uint8_t)value;
    }
    for (int b = 0; b < 64; ++b) {
        int section = b >> 5;
        int local = b & 31;
        int base = section * 128;
        uint32_t value = ((((uint32_t)levels[base + local] & 63u) >> 4) & 3u) |
                         (((((uint32_t)levels[base + local + 32] & 63u) >> 4) & 3u) << 2) |
                         (((((uint32_t)levels[base + local + 64] & 63u) >> 4) & 3u) << 4) |
                         (((((uint32_t)levels[base + local + 96] & 63u) >> 4) & 3u) << 6);
        out[128 + b] = (uint8_t)value;
    }
    for (int g = 0; g < 16; ++g) out[192 + g] = (uint8_t)(scale_codes[g] & 255);
    uint16_t dh = f32_to_f16_bits(d_scale);
    out[208] = (uint8_t)(dh & 0xffu);
    out[209] = (uint8_t)(dh >> 8);
}

int t2c_oracle_quantize_q6_k(const float *x, int64_t rows, int64_t k, uint8_t *out) {
    if (rows < 0 || k < 0 || (k % 256) != 0) return -1;
    int64_t nb = k / 256;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            q6_k_block(x + r * k + b * 256, out + (r * nb + b) * 210);
        }
    }
    return 0;
}

/* ------------------------------------------------------------- decoders --- */
/* embedding_q4_k_f32.py:78-110: w = d*sc*q - dmin*m, evaluated ((d*sc)*q) - (dmin*m) */
int t2c_oracle_dequantize_q4_k(const uint8_t *in, int64_t rows, int64_t k, float *out) {
    if (rows < 0 || k < 0 || (k % 256) != 0) return -1;
    int64_t nb = k / 256;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t *blk = in + (r * nb + b) * 144;
            float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            for (int j = 0; j < 8; ++j) {
                uint32_t sc, m;
                if (j < 4) {
                    sc = blk[4 + j] & 63u;
                    m = blk[8 + j] & 63u;
                } else {
                    sc = (blk[12 + j - 4] & 15u) | ((blk[4 + j - 4] >> 6) << 4);
                    m = (blk[12 + j - 4] >> 4) | ((blk[8 + j - 4] >> 6) << 4);
                }
                float ds = d * (float)sc;
                float dm = dmin * (float)m;
                for (int l = 0; l < 32; ++l) {
                    int idx = 32 * j + l;
                    uint8_t byte = blk[16 + (idx >> 6) * 32 + (idx & 31)];
                    uint32_t q = (idx & 32) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 15u);
                    out[r * k + b * 256 + idx] = ds * (float)q - dm;
                }
            }
        }
    }
    return 0;
}

/* linear_nobias_q6_k_matvec_f32.py:116-156: w = (d*sc)*(L-32) */
int t2c_oracle_dequantize_q6_k(const uint8_t *in, int64_t rows, int64_t k, float *out) {
    if (rows < 0 || k < 0 || (k % 256) != 0) return -1;
    int64_t nb = k / 256;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t *blk = in + (r * nb + b) * 210;
            float d = f16_bits_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
            for (int idx = 0; idx < 256; ++idx) {
                int s = idx >> 7;
                int rem = idx & 127;
                int c = rem >> 5;
                int l = rem & 31;
                uint8_t qlb = blk[64 * s + 32 * (c & 1) + l];
                uint32_t lo = (c >> 1) ? (uint32_t)(qlb >> 4) : (uint32_t)(qlb & 15u);
                uint32_t hi = ((uint32_t)blk[128 + 32 * s + l] >> (2 * c)) & 3u;
                int32_t level = (int32_t)(lo | (hi << 4)) - 32;
                float sc = (float)(int8_t)blk[192 + (idx >> 4)];
                out[r * k + b * 256 + idx] = (d * sc) * (float)level;
            }
        }
    }
    return 0;
}

/* linear_nobias_q8_0_matvec_f32.py:84-95: w = d*q */
int t2c_oracle_dequantize_q8_0(const uint8_t *in, int64_t rows, int64_t k, float *out) {
    if (rows < 0 || k < 0 || (k % 32) != 0) return -1;
    int64_t nb = k / 32;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t *blk = in + (r * nb + b) * 34;
            float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int i = 0; i < 32; ++i) {
                out[r * k + b * 32 + i] = d * (float)(int8_t)blk[2 + i];
            }
        }
    }
    return 0;
}

/* --------------------------------------------------- direct block matvec --- */
/*
 * y[m,n] = sum_k x[m,k] * deq(W)[n,k] with fp16 x, double accumulation, one
 * decoded row at a time: the CPU baseline "direct block matvec" and a fast
 * checker for large N.  type: 0 = Q4_K, 1 = Q6_K, 2 = Q8_0.
 */
int t2c_oracle_matvec(int type, const uint8_t *w, const uint16_t *x, int64_t m, int64_t n, int64_t k,
                      float *y, int64_t row_begin, int64_t row_end) {
    int64_t row_bytes;
    if (type == 0) row_bytes = k / 256 * 144;
    else if (type == 1) row_bytes = k / 256 * 210;
    else if (type == 2) row_bytes = k / 32 * 34;
    else return -1;
    float *row = (float *)malloc((size_t)k * sizeof(float));
    if (row == NULL) return -2;
    for (int64_t r = row_begin; r < row_end && r < n; ++r) {
        const uint8_t *wr = w + r * row_bytes;
        int rc = type == 0 ? t2c_oracle_dequantize_q4_k(wr, 1, k, row)
               : type == 1 ? t2c_oracle_dequantize_q6_k(wr, 1, k, row)
                           : t2c_oracle_dequantize_q8_0(wr, 1, k, row);
        if (rc) {
            free(row);
            return rc;
        }
        for (int64_t t = 0; t < m; ++t) {
            double acc = 0.0;
            const uint16_t *xt = x + t * k;
            for (int64_t i = 0; i < k; ++i) acc += (double)row[i] * (double)f16_bits_to_f32(xt[i]);
            y[t * n + r] = (float)acc;
        }
    }
    free(row);
    return 0;
}

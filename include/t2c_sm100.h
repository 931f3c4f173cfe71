/*
 * t2c_sm100.h -- C ABI of libt2c_sm100.so, the sm_100a (B200) kernels behind
 * torch2vk's quantized-inference hot path.
 *
 * Every entry point:
 *   - takes plain device pointers, element counts and a CUDA stream
 *     (cudaStream_t passed as void*; NULL = legacy default stream);
 *   - launches asynchronously on that stream and never synchronises, never
 *     allocates and never frees device memory (scratch comes from the caller);
 *   - returns T2C_OK (0) or a T2C_E* status; t2c_last_error() then holds a
 *     message for the calling thread.
 *
 * Tensor conventions follow the torch2vk shader contracts: activations are
 * fp16 (IEEE binary16) row-major, weights are the GGUF packed blocks exactly
 * as the reference quantizer writes them (Q4_K: 144 B per 256 values, Q6_K:
 * 210 B per 256, Q8_0: 34 B per 32), norm weights are fp32.
 *
 * Citations name the torch2vk file:line whose shader contract each entry point
 * replaces (paths inside the torch2vk project).
 */
#ifndef T2C_SM100_H
#define T2C_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    T2C_OK = 0,
    T2C_EINVAL = 1,      /* bad shape, pointer, alignment or argument */
    T2C_EUNSUPPORTED = 2,/* valid but not implemented for these sizes/layouts */
    T2C_ECUDA = 3,       /* a CUDA runtime call failed (launch, attribute) */
    T2C_ETIMEOUT = 4,    /* a bounded device-side wait ran out */
    T2C_ESCRATCH = 5     /* caller-provided workspace too small */
};

/* Weight block formats (GGUF ggml type ids). */
enum { T2C_Q8_0 = 8, T2C_Q4_K = 12, T2C_Q6_K = 14, T2C_F16 = 1 };

const char *t2c_last_error(void);
int t2c_abi_version(void);
/* Number of SMs of the current device (grid sizing helper for callers). */
int t2c_device_sm_count(void);

/* ------------------------------------------------------------------ linear
 * y[m, n] = sum_k x[m, k] * deq(W)[n, k]  (+ residual[m, n])
 * x fp16 [M, K]; W packed [N, row_bytes]; y fp16 [M, N]; fp32 accumulation.
 * Replaces, by weight type (run_quantized_linear, src/torch2vk/runtime/quantized_dispatch.py:15-35):
 *   linear_nobias_q4_k_matvec_f32  src/models/quantized_qwen3/shaders/linear_nobias_q4_k_matvec_f32.py:26-197 (M <= 8)
 *   linear_nobias_q4_k_f32         src/models/quantized_qwen3/shaders/linear_nobias_q4_k_f32.py:27-296       (M > 8)
 *   linear_nobias_q6_k_matvec_f32  src/models/quantized_qwen3/shaders/linear_nobias_q6_k_matvec_f32.py:26-193
 *   linear_nobias_q6_k_f32         src/models/quantized_qwen3/shaders/linear_nobias_q6_k_f32.py:27-269
 *   linear_nobias_q8_0_matvec_f32  src/models/quantized_qwen3/shaders/linear_nobias_q8_0_matvec_f32.py:26-119
 *   linear_nobias_q8_0_f32         src/models/quantized_qwen3/shaders/linear_nobias_q8_0_f32.py:27-209
 *   linear_nobias_q{4,6}_k_matvec_add_f32 (residual != NULL)
 *                                  src/models/optimized_qwen3/shaders/linear_nobias_q4_k_matvec_add_f32.py:45-97
 * K must be a multiple of 256 (Q4_K, Q6_K) or 32 (Q8_0).  residual may be NULL
 * and may alias y.
 */
int t2c_linear(int wtype, const void *x, const void *w, const void *residual, void *y,
               int64_t M, int64_t N, int64_t K, void *stream);

/*
 * Fused multi-output matvec: one x, up to three weight streams of possibly
 * different types, each with its own output (and optional residual).
 * Replaces LinearNobiasQ4KQKVMatvecProgram / LinearNobiasQ4QKQ6VMatvecProgram /
 * LinearNobiasQ4KQKMatvecProgram
 *   src/models/optimized_qwen3/shaders/linear_nobias_q4_k_qkv_matvec_f32.py:22-428
 *   src/models/optimized_qwen3/shaders/linear_nobias_q4_qk_q6_v_matvec_f32.py:103-162
 *   src/models/optimized_qwen3/shaders/linear_nobias_q4_k_qk_matvec_f32.py:22-315
 * norm_weight (fp32 [K]) may be non-NULL: the kernel then applies RMSNorm
 * (eps) to x before the product (rms_norm_mul_f16_f32 fused as a prologue).
 */
int t2c_linear_multi(int count, const int *wtypes, const void *const *ws, void *const *ys,
                     const void *const *residuals, const int64_t *Ns, const void *x,
                     const float *norm_weight, float eps, int64_t M, int64_t K, void *stream);

/*
 * Gate/up pair with the SwiGLU epilogue: y[m, n] = silu(x.Wg[n]) * (x.Wu[n]).
 * Replaces the gate+up matvec + swiglu_f16 pair
 *   src/models/optimized_qwen3/shaders/linear_nobias_q4_k_qk_matvec_f32.py:22-315
 *   src/models/optimized_qwen3/shaders/swiglu_f16.py:20-80
 * norm_weight as in t2c_linear_multi.
 */
int t2c_linear_swiglu(int wtype, const void *x, const void *w_gate, const void *w_up, void *y,
                      const float *norm_weight, float eps, int64_t M, int64_t N, int64_t K,
                      void *stream);

/* ------------------------------------------------------------- quantizers
 * fp32 [R, K] -> packed blocks, bit-exact with the reference quantizer's
 * arithmetic (src/torch2vk/quantize/vulkan.py:91-185 Q8_0, :188-419 Q4_K,
 * :422-637 Q6_K).  out must hold R * row_bytes bytes.
 */
int t2c_quantize(int wtype, const float *x, void *out, int64_t R, int64_t K, void *stream);
/* packed blocks -> fp32 [R, K] (decoders of the same shader files). */
int t2c_dequantize(int wtype, const void *w, float *out, int64_t R, int64_t K, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* T2C_SM100_H */

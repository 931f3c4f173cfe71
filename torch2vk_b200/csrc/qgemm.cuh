// Quantized GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) for
// M > 4 tokens: y[m, n] = sum_k x[m, k] * deq(W)[n, k] (+ residual), or the
// SwiGLU of two weights.  Internal interface between qlinear.cu and qgemm.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cuda_fp16.h>

namespace t2c {

struct QGemmArgs {
    int fmt;               // T2C_Q4_K, T2C_Q6_K (K a multiple of 2048) or T2C_Q8_0 (K a multiple of 256); SwiGLU Q4_K only
    int nw;                // weights sharing x (1..3: fused QKV), 1 with SwiGLU
    const uint8_t *w[3];   // Q4_K rows (row_bytes = K / 256 * 144), 16-byte aligned
    const uint8_t *w_up;   // SwiGLU: the up weight (same shape as w[0]), else nullptr
    int64_t N[3], K, M;
    const __half *x;       // [M, K], 16-byte aligned rows
    __half *y[3];          // [M, N[i]]
    float *yf[3];          // fp32 [M, N[i]] written instead of y[i] when non-null (no residual / SwiGLU)
    const __half *res[3];  // [M, N[i]] or nullptr
    float *ps;             // argmax mode (LM head): best (score, row) per 4 rows [M, G], else nullptr
    uint32_t *pt;
    int64_t G;
    const float *bias;     // fp32 [N] added before the activation (one plain weight), or nullptr
    int act;               // 1: erf GELU after the bias (one plain weight)
};

// Returns T2C_OK, or T2C_EUNSUPPORTED when the shape is not served (caller falls back).
int qgemm(const QGemmArgs &a, cudaStream_t stream);
// 5.. tokens of Q4_K weights, 16 per launch (qbatch.cu): exact fp16-x batched matvec, optional fused RMSNorm.
int qbatch(const QGemmArgs &a, const float *norm_w, float eps, cudaStream_t stream);
cudaError_t status_qbatch(unsigned int *bits, int clear, cudaStream_t s);
cudaError_t status_qgemm(unsigned int *bits, int clear, cudaStream_t s);

}  // namespace t2c

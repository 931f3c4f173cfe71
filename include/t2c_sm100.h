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
enum { T2C_Q8_0 = 8, T2C_Q4_K = 12, T2C_Q6_K = 14, T2C_F16 = 1, T2C_F32 = 0 };

const char *t2c_last_error(void);
int t2c_abi_version(void);
/* Reads (and with clear != 0 resets) the device status bits that kernels set
 * with 1 << T2C_E* (e.g. T2C_ETIMEOUT when a bounded wait ran out).  Synchronises
 * the stream. */
int t2c_device_status(unsigned int *bits, int clear, void *stream);
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

/*
 * LM head with the greedy-select partial epilogue: for every token m and every
 * group of 4 consecutive vocabulary rows g, partial_scores[m, g] / partial_tokens[m, g]
 * hold the best fp32 logit and its row (ties -> lower row), G = ceil(N / 4).
 * Replaces LmHeadQ6KArgmaxPartialF16Program
 *   src/torch2vk/export/shaders/lm_head_q6_k_argmax_partial_f16.py (batch 1 there;
 *   here M tokens).  norm_weight as in t2c_linear_multi (final RMSNorm fused).
 */
int t2c_lm_head_argmax(int wtype, const void *x, const void *w, float *partial_scores,
                       uint32_t *partial_tokens, const float *norm_weight, float eps, int64_t M,
                       int64_t N, int64_t K, void *stream);

/* ---------------------------------------------------------- greedy select
 * Reduces G partials per token to the winning token (ties -> lower id) and
 * flags it done when it equals one of the E eos ids.
 * Replaces Qwen3TokenSelectReduceF32Program / Qwen3TokenSelectReduceChunksF32Program
 *   src/torch2vk/export/shaders/qwen3_token_select_reduce_f32.py:21-241
 * partial_* are [M, G]; next_token int64 [M]; done uint32 [M].
 */
int t2c_token_select(const float *partial_scores, const uint32_t *partial_tokens, int64_t M, int64_t G,
                     const int64_t *eos_ids, int64_t E, int64_t *next_token, uint32_t *done, void *stream);

/*
 * Appends next_token[b] at generated_tokens[b, token_index] (capacity G) and
 * updates generated_length / stopped, honouring stop_on_eos.  token_index is
 * read from device memory (token_index_dev, int32) when non-NULL so a
 * captured graph can replay it, else taken from token_index.
 * Replaces Qwen3TokenStoreEosProgram / Qwen3TokenStoreProgram
 *   src/torch2vk/export/shaders/qwen3_token_store.py:1-145
 */
int t2c_token_store(const int64_t *next_token, const uint32_t *done, int64_t *generated_tokens,
                    uint32_t *generated_length, uint32_t *stopped, int64_t B, int64_t G, int32_t token_index,
                    const int32_t *token_index_dev, int stop_on_eos, void *stream);

/* ------------------------------------------------------------------ norms
 * y = fp16(x * rsqrt(mean(x^2) + eps) * w); x, y fp16 [rows, cols], w fp32 [cols].
 * Replaces ExportRmsNormF32WeightProgram / OptimizedQwen3RmsNormMulF16F32Program
 *   src/models/quantized_qwen3/shaders/rms_norm_f32w_f32.py:21-94
 *   src/models/optimized_qwen3/shaders/rms_norm_mul_f16_f32.py:22-115
 */
int t2c_rms_norm(const void *x, const float *w, void *y, int64_t rows, int64_t cols, float eps, void *stream);

/*
 * Fused per-head RMSNorm (q_norm / k_norm) + rotate-half RoPE + cache write
 * for one attention layer, M = B * T tokens:
 *   q[m, h, :]  <- rope(rmsnorm(q_in[m, h, :]) * q_w)          (h < NH)
 *   k_cache[b, pos, kh, :] <- rope(rmsnorm(k_in[m, kh, :]) * k_w)
 *   v_cache[b, pos, kh, :] <- v_in[m, kh, :]
 * with pos = positions[b] + t, angle_i = pos * inv_freq[i] (fp32, i < D/2; the
 * caller supplies inv_freq[i] = theta^(-2 i / D) as its model computes it).
 * Caches are addressed by element strides (batch, position, head) so both
 * the head-major [B, NK, S, D] and token-major [B, S, NK, D] layouts work.
 * q_out may alias q_in.  Replaces the q/k-norm + RoPE + cache-write chain
 *   src/models/optimized_qwen3/shaders/rms_norm_rope_transpose_f16.py:22-146,
 *   rms_norm_rope_token_f32.py:22, token_major_kv_cache_write_f16_pair.py:20-105,
 *   src/models/quantized_qwen3/shaders/kv_cache_write_f16.py:22-92, src/torch2vk/runtime/rope_table.py:31-121
 */
int t2c_qk_norm_rope_cache(const void *q_in, const void *k_in, const void *v_in, const float *q_w,
                           const float *k_w, void *q_out, void *k_cache, void *v_cache,
                           const int32_t *positions, int64_t B, int64_t T, int64_t NH, int64_t NK, int64_t D,
                           int64_t cache_b_stride, int64_t cache_s_stride, int64_t cache_h_stride,
                           const float *inv_freq, float eps, void *stream);

/* ------------------------------------------------------------- attention
 * Decode attention (one query token per batch row) over a KV cache:
 * out[b, h, :] = softmax(q[b, h] . K[b, 0..len_b)^T / sqrt(D)) V, GQA
 * kv head = h / (NH / NK), len_b = positions[b] + 1.  Split-K over cache
 * positions in `splits` parts (max_len / splits positions each); the partial
 * (max, sum, acc) go to `workspace` (fp32, B * NH * splits * (D + 2) floats,
 * caller-provided; unused when splits == 1) and a combine pass writes out.
 * A position outside [0, max_len) sets T2C_EINVAL in the device status word
 * (t2c_device_status) and its rows attend to nothing (zero output).
 * Replaces ExportSdpaDecodeCacheF16Program / SdpaDecodeCacheWriteF32Program
 *   src/models/quantized_qwen3/shaders/sdpa_decode_cache_f16.py:22-136
 *   src/models/optimized_qwen3/shaders/sdpa_decode_cache_write_f32.py:22-171
 */
int t2c_attn_decode(const void *q, const void *k_cache, const void *v_cache, void *out,
                    const int32_t *positions, int64_t B, int64_t NH, int64_t NK, int64_t D, int64_t max_len,
                    int64_t cache_b_stride, int64_t cache_s_stride, int64_t cache_h_stride, int64_t splits,
                    float *workspace, int64_t workspace_floats, void *stream);

/*
 * One decode step of attention in one launch (T = 1 query per batch row):
 * q / k RMSNorm (fp32 weights q_w / k_w [D]) and RoPE (inv_freq [D/2]) of the
 * raw projections, the new k / v written into the caches at positions[b],
 * split-K attention over cache positions 0..positions[b] and the split
 * combine.  Replaces the chain rms_norm_rope_transpose_f16 ->
 * token_major_kv_cache_write_f16_pair -> sdpa_decode_cache_write_f32
 * (src/models/optimized_qwen3/dispatch/decode_layer.py:36-128) and
 * sdpa_decode_cache_f16.py:22-136.  q_in [B, NH*D], k_in / v_in [B, NK*D] with
 * batch strides q_sb / k_sb / v_sb (elements); out [B, NH*D] with o_sb.  D = 128.
 * max_len: cache rows per sequence; a position outside [0, max_len) makes the
 * kernel touch nothing and set T2C_EINVAL in t2c_device_status.
 * splits <= 8: the splits CTAs of one (b, kv head) form a thread-block
 * cluster and combine through distributed shared memory (no workspace).
 * splits > 8 needs t2c_attn_decode_fused_workspace(...) words of workspace whose
 * last B*NH words (arrival counters) are zero before the first call; every
 * call leaves them zero.  positions, q_w, k_w, inv_freq and the cache rows of
 * earlier positions are read before the wait on the preceding kernel of the
 * stream, so they must not be written by that kernel (positions advanced one
 * launch earlier or by a copy are fine).
 */
int t2c_attn_decode_fused(const void *q_in, const void *k_in, const void *v_in, int64_t q_sb, int64_t k_sb,
                          int64_t v_sb, const float *q_w, const float *k_w, const float *inv_freq, float eps,
                          void *k_cache, void *v_cache, int64_t cache_b_stride, int64_t cache_s_stride,
                          int64_t cache_h_stride, void *out, int64_t o_sb, const int32_t *positions, int64_t B,
                          int64_t NH, int64_t NK, int64_t D, int64_t max_len, int64_t splits, float *workspace,
                          int64_t workspace_floats, void *stream);
int64_t t2c_attn_decode_fused_workspace(int64_t B, int64_t NH, int64_t NK, int64_t D, int64_t splits);

/*
 * Paged KV cache (split-K decode attention and the cache write).  The cache is
 * a pool of pages, each page_size (a power of two) positions of NK heads x D
 * fp16: element (page, row, head, d) at page * page_stride + row * row_stride
 * + head * head_stride + d.  block_table[b * bt_stride + i] is the physical
 * page holding positions [i * page_size, (i + 1) * page_size) of sequence b,
 * so a sequence holds at most bt_stride * page_size positions.  Attention is
 * t2c_attn_decode's (same workspace rule, output layout and out-of-range
 * position report) with the row address taken from the table; the write
 * stores T new rows per sequence (src [B, T, NK * D] by element strides) at
 * positions[b] .. positions[b] + T - 1.  A table entry outside
 * [0, num_pages) is reported through t2c_device_status (the write skips that
 * row; attention reads page 0 in its place).
 * The reference keeps one contiguous cache per layer (kv_cache_write_f16.py:22-92,
 * sdpa_decode_cache_f16.py:22-136); the paged layout serves the same attention
 * contract for many sequences sharing one pool.
 */
int t2c_attn_decode_paged(const void *q, const void *k_pages, const void *v_pages, void *out,
                          const int32_t *positions, const int32_t *block_table, int64_t bt_stride, int64_t num_pages,
                          int64_t page_size, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                          int64_t B, int64_t NH, int64_t NK, int64_t D, int64_t splits, float *workspace,
                          int64_t workspace_floats, void *stream);
int t2c_kv_cache_write_paged(void *pages, const void *src, int64_t src_b_stride, int64_t src_t_stride,
                             const int32_t *positions, const int32_t *block_table, int64_t bt_stride,
                             int64_t num_pages, int64_t page_size, int64_t page_stride, int64_t row_stride,
                             int64_t head_stride, int64_t B, int64_t T, int64_t NK, int64_t D, void *stream);

/*
 * t2c_attn_decode for callers that cannot allocate device memory: the same
 * split-K decode attention, with its split partials kept in a fixed 16 MiB
 * device array inside the library instead of a caller workspace.  Meant for
 * hosts that own every device allocation themselves and forbid a plugin to
 * call cudaMalloc (fixed-budget serving executors, embedding runtimes that
 * pre-plan all memory, code that runs where allocation is not allowed).
 * This entry point has no counterpart in the reference (its shaders receive
 * all scratch as bound buffers).
 *   - Limit: B * NH * splits * (D + 2) <= 4194304 floats, else T2C_ESCRATCH
 *     (splits == 1 needs no scratch).
 *   - Allocates nothing: no cudaMalloc / cudaFree / allocating library call.
 *     The array exists on every GPU that loads the library, until exit.
 *   - The first call on a device resolves the array's device address on the
 *     current device (cudaGetSymbolAddress); make that first call before any
 *     stream capture.  The address is kept for the device's primary context:
 *     do not call again on a device after cudaDeviceReset.
 *   - Shape checks come first (T2C_EINVAL / T2C_EUNSUPPORTED for splits > 64
 *     or head_dim other than 64 / 128), then the scratch limit.
 *   - All calls share the one array, which keeps the last call's contents;
 *     every split record is fully rewritten before it is read, so nothing
 *     needs clearing, but calls that overlap on the GPU (other streams or
 *     threads) race on it and must be serialised by the caller.
 */
int t2c_attn_decode_static(const void *q, const void *k_cache, const void *v_cache, void *out,
                           const int32_t *positions, int64_t B, int64_t NH, int64_t NK, int64_t D, int64_t max_len,
                           int64_t cache_b_stride, int64_t cache_s_stride, int64_t cache_h_stride, int64_t splits,
                           void *stream);

/*
 * Causal prefill attention: T queries per batch row, keys/values read from
 * the caches for positions 0 .. positions[b] + T - 1 (the current chunk
 * already written); query t of batch b attends to cache positions
 * <= positions[b] + t.  q and out are addressed by element strides
 * (batch, token, head): token-major [B, T, NH, D] or head-major [B, NH, T, D].
 * Replaces ExportSdpaProgram (causal)
 *   src/models/quantized_qwen3/shaders/sdpa_causal_f32.py:22-142
 */
int t2c_attn_prefill(const void *q, const void *k_cache, const void *v_cache, void *out,
                     const int32_t *positions, int64_t B, int64_t T, int64_t NH, int64_t NK, int64_t D,
                     int64_t cache_b_stride, int64_t cache_s_stride, int64_t cache_h_stride, int64_t q_b_stride,
                     int64_t q_t_stride, int64_t q_h_stride, int64_t out_b_stride, int64_t out_t_stride,
                     int64_t out_h_stride, void *stream);

/* ---------------------------------------------------- exported-graph ops
 * Strided 4-D copy dst[i] = src[i] (element size 1/2/4/8 bytes; strides in
 * elements).  Serves the slice / cat / transpose / contiguous-view contracts
 * (ExportSliceProgram, ExportCat2Program, ExportTransposeProgram,
 *  SliceLastTokenF16Program) of src/models/quantized_qwen3/shaders/{slice_f32,
 *  cat_2_f32,transpose_f32_*,slice_last_token_f16}.py.
 */
int t2c_copy4d(int elem_bytes, const void *src, const int64_t *src_strides, void *dst, const int64_t *dst_strides,
               const int64_t *shape, void *stream);
/*
 * Broadcasting 4-D elementwise op (0 add, 1 mul, 2 neg, 3 silu) on fp16
 * (is_f32 = 0) or fp32 tensors; zero strides broadcast.  Serves
 * ExportAddF32Program, ExportMulF32Program, ExportMulBroadcastProgram,
 * ExportNegF32Program, ExportSiluF32Program (src/models/quantized_qwen3/shaders/).
 */
int t2c_elementwise4d(int op, int is_f32, const void *a, const int64_t *a_strides, const void *b,
                      const int64_t *b_strides, void *out, const int64_t *out_strides, const int64_t *shape,
                      void *stream);
/* RoPE cos/sin tables [B, T, D] fp16 (src/torch2vk/runtime/rope_table.py:31-121). */
int t2c_rope_table(void *cos_out, void *sin_out, int64_t B, int64_t T, int64_t D, float theta,
                   int64_t start_position, float attention_scaling, void *stream);
/* The same table in fp32.  Replaces RopeTableOutputF32Program
 *   src/torch2vk/runtime/rope_table.py:124-160 */
int t2c_rope_table_f32(float *cos_out, float *sin_out, int64_t B, int64_t T, int64_t D, float theta,
                       int64_t start_position, float attention_scaling, void *stream);
/* The same tables (fp16, or fp32 when out_f32) with the start position read from device
 * memory (int64), so a captured CUDA graph replays them at each step's position.  Replaces the
 * push-constant input start_position of RopeTableF32Program / RopeTableOutputF32Program under
 * replay (src/torch2vk/runtime/rope_table.py:31-160, src/torch2vk/runtime/replay.py:163-364). */
int t2c_rope_table_dev(void *cos_out, void *sin_out, int64_t B, int64_t T, int64_t D, float theta,
                       const int64_t *start_position_dev, float attention_scaling, int out_f32, void *stream);
/*
 * Per-row RMSNorm + rotate-half RoPE from fp16 cos/sin tables [B, T, D]; x
 * [B, T, G, D] fp16, out addressed by strides (b, g, t).  Replaces
 * OptimizedQwen3RmsNormRopeTransposeF16Program
 *   src/models/optimized_qwen3/shaders/rms_norm_rope_transpose_f16.py:22-146
 */
int t2c_rms_norm_rope(const void *x, const float *w, const void *cos_t, const void *sin_t, void *out, int64_t B,
                      int64_t T, int64_t G, int64_t D, int64_t out_b_stride, int64_t out_g_stride,
                      int64_t out_t_stride, float eps, void *stream);
/*
 * cache[b, pos, h, :] = src[b, t, h, :] with pos = positions[t] (int64 [T]) or,
 * when positions is NULL, position + t; cache of S positions, both addressed
 * by element strides.  Replaces ExportKvCacheWriteF16Program (both variants)
 * and the token-major pair/triple writes
 *   src/models/quantized_qwen3/shaders/kv_cache_write_f16.py:22-92, kv_cache_write_decode_f16.py:23-85
 *   src/models/optimized_qwen3/shaders/token_major_kv_cache_write_f16_pair.py:20-105
 */
int t2c_kv_cache_write(void *cache, const void *src, const int64_t *positions, int64_t position, int64_t B,
                       int64_t H, int64_t T, int64_t D, int64_t S, int64_t cache_b_stride, int64_t cache_s_stride,
                       int64_t cache_h_stride, int64_t src_b_stride, int64_t src_t_stride, int64_t src_h_stride,
                       void *stream);
/* Best (score, token) per chunk of 1024 partials (ties -> lower token); C = ceil(G / 1024) outputs.
 * Replaces Qwen3TokenSelectReduceChunksF32Program (qwen3_token_select_reduce_f32.py:21-148). */
int t2c_token_select_chunks(const float *scores, const uint32_t *tokens, int64_t G, float *chunk_scores,
                            uint32_t *chunk_tokens, void *stream);

/* ---------------------------------------------------------------- misc
 * Embedding gather: out[i, :] = deq(weight[ids[i], :]) for F16 or Q4_K rows.
 * Replaces ExportEmbeddingQ4_KProgram
 *   src/models/quantized_qwen3/shaders/embedding_q4_k_f32.py:25-121
 */
int t2c_embedding(int wtype, const void *weight, const int64_t *ids, void *out, int64_t n_ids, int64_t vocab,
                  int64_t H, void *stream);
/* y = x + r (fp16, n elements).  Replaces ExportAddF32Program (add_f32*.py). */
int t2c_add(const void *x, const void *r, void *y, int64_t n, void *stream);
/* y = fp16(silu(g)) * u (fp16).  Replaces OptimizedQwen3SwiGLUF16Program
 *   src/models/optimized_qwen3/shaders/swiglu_f16.py:20-80 */
int t2c_swiglu(const void *g, const void *u, void *y, int64_t n, void *stream);

/*
 * End-of-step bookkeeping for a captured decode graph: positions[b] += 1 for
 * b < B and *token_index += 1 (both int32, device memory).  Replaces the
 * host-side push-constant updates of the reference replay loop
 *   src/torch2vk/runtime/replay.py:321 (stage_replay_step_inputs) /
 *   src/models/quantized_qwen3/run.py:357-388
 */
int t2c_advance_positions(int32_t *positions, int64_t B, int32_t *token_index, void *stream);

/* ------------------------------------------------------------- quantizers
 * fp32 [R, K] -> packed blocks, bit-exact with the reference quantizer's
 * arithmetic (src/torch2vk/quantize/vulkan.py:91-185 Q8_0, :188-419 Q4_K,
 * :422-637 Q6_K).  out must hold R * row_bytes bytes.
 */
int t2c_quantize(int wtype, const float *x, void *out, int64_t R, int64_t K, void *stream);
/* packed blocks -> fp32 [R, K] (decoders of the same shader files). */
int t2c_dequantize(int wtype, const void *w, float *out, int64_t R, int64_t K, void *stream);

/* ------------------------------------------------------------------ ASR audio encoder
 * Qwen3-ASR audio tower (models/quantized_qwen3_asr/dispatch/audio_encoder.py): Q8_0 weights,
 * fp16 activations, fp32 biases.
 *
 * y[M, N] = x[M, K] @ deq(W)^T + bias (bias may be NULL; act 1 applies GELU (erf) after the
 * bias).  W: Q8_0 rows of ceil(K/32) blocks.  x 16-byte aligned, K a multiple of 8.
 * Replaces ExportLinearBiasQ8_0WeightF32BiasProgram
 *   src/models/quantized_qwen3_asr/shaders/linear_bias_q8_0w_f32b_f32.py:38-92
 * and (bias NULL) ExportLinearNobiasQ8_0Program (linear_nobias_q8_0_f32.py).
 */
int t2c_linear_q8_0_bias(const void *x, const void *w, const float *bias, void *y, int64_t M, int64_t N, int64_t K,
                         int act, void *stream);
/* NCHW fp16 conv2d with Q8_0 weights [Co, ceil(Ci*kh*kw / 32) blocks] (k = (ic, fh, fw)), fp32
 * bias, zero padding; out [B, Co, Ho, Wo]; act 1 applies GELU after the bias.
 * Replaces ExportConv2dQ8_0WeightF32BiasProgram
 *   src/models/quantized_qwen3_asr/shaders/conv2d_q8_0w_f32b_f16.py:36-98 */
int t2c_conv2d_q8_0(const void *x, const void *w, const float *bias, void *out, int64_t B, int64_t Ci, int64_t Hi,
                    int64_t Wi, int64_t Co, int64_t Ho, int64_t Wo, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                    int64_t ph, int64_t pw, int act, void *stream);
/* The same convolution writing channels-last output [B, Ho, Wo, Co] (the layout the next
 * convolution's 16-byte im2col gathers read; the ASR tower's first convolution). */
int t2c_conv2d_q8_0_nhwc(const void *x, const void *w, const float *bias, void *out, int64_t B, int64_t Ci,
                         int64_t Hi, int64_t Wi, int64_t Co, int64_t Ho, int64_t Wo, int64_t kh, int64_t kw,
                         int64_t sh, int64_t sw, int64_t ph, int64_t pw, int act, void *stream);
/* im2col of a 2-D convolution for the tensor-core GEMM: cols [B*Ho*Wo, Kp] fp16 (16-byte aligned),
 * row (b, oh, ow), column (c, i, j) = x[b, c, oh*sh - ph + i, ow*sw - pw + j] (zero outside), columns
 * C*kh*kw .. Kp - 1 zero (Kp a multiple of 8).  x fp16 read through element strides
 * x_strides = {b, c, h, w} (host array): NCHW, or the [B, Ho, Wo, C] rows a GEMM wrote.
 * channels_last = 1 states that x has unit channel stride: for a 3 x 3 kernel with C % 8 == 0 and
 * 16-byte aligned pixels the columns (same order) are then gathered by 16-byte loads of 8 channels.
 * With the weights padded to Kp columns, t2c_linear_q8_0_bias(cols, ...) is the convolution with
 * NHWC output (the ASR tower's 480-channel convolutions: conv2d_q8_0w_f32b_f16.py:36-98). */
int t2c_im2col_f16(const void *x, void *cols, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ho, int64_t Wo,
                   int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t Kp,
                   const int64_t *x_strides, int channels_last, void *stream);
/* Row LayerNorm, fp16 x / y [rows, cols], fp32 w / b [cols] (cols a multiple of 8, <= 4096).
 * Replaces ExportLayerNormF32WeightF32BiasProgram (layer_norm_f32w_f32b_f32.py). */
int t2c_layer_norm(const void *x, const float *w, const float *b, void *y, int64_t rows, int64_t cols, float eps,
                   void *stream);
/* The same LayerNorm into rows of y_cols >= cols halves (a multiple of 8), columns cols .. y_cols - 1
 * written as zeros: the zero-padded K of the next tcgen05 GEMM's input (the ASR tower's d_model 896
 * linears padded to K = 1024) without a separate fill and copy.  No counterpart in the reference. */
int t2c_layer_norm_padded(const void *x, const float *w, const float *b, void *y, int64_t rows, int64_t cols,
                          int64_t y_cols, float eps, void *stream);
/* y = x * 0.5 * (1 + erf(x / sqrt 2)), fp16.  Replaces ExportGeluF32Program (gelu_f32.py). */
int t2c_gelu(const void *x, void *y, int64_t n, void *stream);
/* out[o, :] = x[index[o], :] (fp16 rows of H; int64 index; an index outside [0, rows) writes a
 * zero row and sets T2C_EINVAL).  Replaces ExportIndexSelectF32Program (index_select_f32_*.py). */
int t2c_index_rows(const void *x, const int64_t *index, void *out, int64_t O, int64_t H, int64_t rows, void *stream);
/* cache[b, index[s], :] = src[b, s, :] (fp16; cache [B, T, H], src [B, S, H]); a row index
 * outside [0, T) is skipped and sets T2C_EINVAL.  Replaces ExportIndexCopyF32Program
 *   src/models/quantized_qwen3_asr/shaders/index_copy_f32_7ba4f1ff13.py (audio-feature injection) */
int t2c_index_copy_rows(void *cache, const int64_t *index, const void *src, int64_t B, int64_t T, int64_t S, int64_t H,
                        void *stream);
/* out fp16 [n_ids, H] = d * q of Q8_0 rows (an id outside [0, vocab) reads row 0 and sets
 * T2C_EINVAL).  Replaces ExportEmbeddingQ8_0Program
 *   src/models/quantized_qwen3_asr/shaders/embedding_q8_0_f32.py */
int t2c_embedding_q8_0(const void *weight, const int64_t *ids, void *out, int64_t n_ids, int64_t vocab, int64_t H,
                       void *stream);
/* Non-causal attention with an additive fp16 mask (the encoder's block-diagonal windows):
 * out[b,h,t,:] = softmax(q[b,h,t,:] . k[b,h,s,:] * scale + mask[b,h,t,s]) v[b,h,s,:], D = 64.
 * Strides (elements) are {batch, head, row} for q, k, v, out and {batch, head, query row} for the
 * mask (0 broadcasts; the key stride is 1).  Replaces ExportSdpaProgram
 *   src/models/quantized_qwen3_asr/shaders/sdpa_masked_f32.py:33-90 */
int t2c_attn_masked(const void *q, const void *k, const void *v, const void *mask, void *out, int64_t B, int64_t H,
                    int64_t T, int64_t S, int64_t D, const int64_t *q_strides, const int64_t *k_strides,
                    const int64_t *v_strides, const int64_t *m_strides, const int64_t *o_strides, float scale,
                    void *stream);

/* ------------------------------------------------------------------ fp32-activation prefill
 * The optimized Qwen3 model's llama.cpp-style prefill chain keeps activations in
 * fp32 between programs (src/models/optimized_qwen3/dispatch/text_layer.py:131-199).
 */
/* y fp32 [M, N] = x fp32 [M, K] @ deq(W)^T.  x is rounded to fp16 into the caller's
 * scratch (t2c_linear_f32_scratch_bytes, 256-byte aligned) and multiplied on the
 * tensor cores with fp32 accumulation; the reference multiplies fp16 operands
 * with fp16 accumulation.  Replaces LlamaMatmulQ4KF32Program / LlamaMatmulQ6KF32Program
 *   src/models/optimized_qwen3/shaders/llama_matmul_q4_k_f32.py:31-141
 *   src/models/optimized_qwen3/shaders/llama_matmul_q6_k_f32.py */
int64_t t2c_linear_f32_scratch_bytes(int64_t M, int64_t N, int64_t K);
int t2c_linear_f32(int wtype, const float *x, const void *w, float *y, int64_t M, int64_t N, int64_t K, void *scratch,
                   int64_t scratch_bytes, void *stream);
/* y = x * rsqrt(mean(x^2) + eps) * w per row, fp32 (x, y [rows, H]; w [H]).  Replaces
 * OptimizedQwen3RmsNormMulF32Program  src/models/optimized_qwen3/shaders/rms_norm_mul_f32.py */
int t2c_rms_norm_f32(const float *x, const float *w, float *y, int64_t rows, int64_t H, float eps, void *stream);
/* RMSNorm (w [D]) + rotate-half RoPE from fp16 cos / sin tables [B, T, D] of fp32
 * x [B, T, G, D]; out [B, T, G, D] fp32 (out_f32 != 0) or fp16.  D = 64 or 128.
 * Replaces OptimizedQwen3RmsNormRopeTokenF32Program / ...F32ToF16Program
 *   src/models/optimized_qwen3/shaders/rms_norm_rope_token_f32.py:22
 *   src/models/optimized_qwen3/shaders/rms_norm_rope_token_f32_to_f16.py */
int t2c_rms_norm_rope_f32(const float *x, const float *w, const void *cos_t, const void *sin_t, void *out, int out_f32,
                          int64_t B, int64_t T, int64_t G, int64_t D, float eps, void *stream);
/* out = a + b (op 0) or silu(a) * b (op 1), fp32, n elements, 16-byte aligned.
 * Replaces AddF32PrefillProgram (add_f32_prefill.py) and SwigluF32Program (swiglu_f32.py). */
int t2c_binary_f32(int op, const float *a, const float *b, float *out, int64_t n, void *stream);
/* y = x converted between T2C_F32 and T2C_F16 (n elements). */
int t2c_cast(const void *x, int x_dtype, void *y, int y_dtype, int64_t n, void *stream);
/* out[b, 0, :] = fp16(x[b, S - 1, :]).  Replaces SliceLastTokenF32ToF16Program
 *   src/models/optimized_qwen3/shaders/slice_last_token_f32_to_f16.py */
int t2c_slice_last_f32_to_f16(const float *x, void *out, int64_t B, int64_t S, int64_t H, void *stream);
/* Token-major fp16 caches[i] [B, cache_lens[i], H, D] (1..3 of them) receive
 * fp16(src[b, t, h, :]) at row positions[t] (int64); a cache too short for the row
 * is skipped, as in the reference.  Replaces
 * OptimizedQwen3TokenMajorValueCacheWriteF32ToF16{Pair,Triple}Program
 *   src/models/optimized_qwen3/shaders/token_major_value_cache_write_f32_to_f16_pair.py */
int t2c_value_cache_write_f32(const float *src, const int64_t *positions, int ncaches, void *const *caches,
                              const int64_t *cache_lens, int64_t B, int64_t T, int64_t H, int64_t D, void *stream);
/* Bidirectional GQA attention under an additive fp16 mask (OmniVoice's LLM):
 * out[b,t,h,:] = softmax(q[b,t,h,:] . k[b,s,h/(NH/NK),:] * scale + mask[b,t,s]) v[b,s,h/(NH/NK),:]
 * over all S keys, fp16 q / k / v / out addressed by element strides {batch, position, head}
 * (k and v share theirs; rows of D contiguous values), mask element (b, t, s) at
 * b * mask_b_stride + t * mask_row_stride + s (values <= -FLT_MAX/2, -inf included, mask the
 * key).  D = 128, on the tensor cores.  Replaces ExportSdpaProgram
 *   src/models/quantized_omnivoice/shaders/sdpa_masked_f32.py */
int t2c_attn_masked_gqa(const void *q, const void *k, const void *v, const void *mask, void *out, int64_t B,
                        int64_t T, int64_t S, int64_t NH, int64_t NK, int64_t D, const int64_t *q_strides,
                        const int64_t *kv_strides, const int64_t *o_strides, int64_t mask_b_stride,
                        int64_t mask_row_stride, float scale, void *stream);
/* OmniVoice input embedding: out fp16 [B, S, H]; where audio_mask[b, s] != 0 the fp32 sum over the C
 * codebooks of Q8_0 audio rows c * audio_vocab + ids[b, c, s], else Q8_0 text row ids[b, 0, s]
 * (ids int64 [B, C, S], audio_mask uint32 [B, S]).  An id outside its table reads row 0 and sets
 * T2C_EINVAL.  Replaces OmniVoiceInputEmbedQ8_0Program
 *   src/models/quantized_omnivoice/custom_shaders.py:17-181 */
int t2c_omnivoice_input_embed(const void *text_weight, const void *audio_weight, const int64_t *ids,
                              const uint32_t *audio_mask, void *out, int64_t B, int64_t C, int64_t S, int64_t H,
                              int64_t text_vocab, int64_t audio_vocab, void *stream);
/* Flash-attention mask classifier: out [row_blocks, words] uint32, 2 bits per
 * (16-row, 64-column) block of the fp16 mask [T, S]: 1 = every value <= -FLT_MAX/2
 * (or outside the mask), 2 = every value 0.  Replaces OptimizedQwen3FaMaskOptF16Program
 *   src/models/optimized_qwen3/shaders/fa_mask_opt_f16.py */
int t2c_fa_mask_opt(const void *mask, uint32_t *out, int64_t T, int64_t S, int64_t words, int64_t row_blocks,
                    void *stream);
/* softmax(q k^T * scale + mask) v over keys [0, S) of token-major fp16 caches
 * [B, S, NK, D]; q and out fp32 token-major [B, T, NH, D]; mask fp16 [T, S]
 * (row stride mask_row_stride); mask_opt (optional, from t2c_fa_mask_opt) lets a
 * warp skip fully masked 64-key tiles.  D = 128, on the tensor cores.  Replaces
 * LlamaFlashAttnF32F16F16Program
 *   src/models/optimized_qwen3/shaders/llama_flash_attn_f32_f16_f16.py:35-158 */
int t2c_attn_prefill_masked_f32(const float *q, const void *k_cache, const void *v_cache, const void *mask,
                                const uint32_t *mask_opt, float *out, int64_t B, int64_t T, int64_t S, int64_t NH,
                                int64_t NK, int64_t D, int64_t mask_row_stride, int64_t mask_opt_row_stride,
                                float scale, void *stream);
/* out fp32 [n_ids, H] = rows of a Q4_K embedding.  Replaces
 * OptimizedQwen3EmbeddingQ4KActF32Program  src/models/optimized_qwen3/shaders/embedding_q4_k_act_f32.py */
int t2c_embedding_f32(int wtype, const void *weight, const int64_t *ids, float *out, int64_t n_ids, int64_t vocab,
                      int64_t H, void *stream);

/* Elementwise steps of the exported (unfused) RMSNorm chain, fp32 arithmetic; a_f16 / b_f16 /
 * out_f16 select fp16 (1) or fp32 (0) storage.  op 0: a*a (ExportPowScalarF32Program, exponent 2),
 * 1: 1/sqrt(a) (ExportRsqrtF32Program), 2: a + scalar (ExportAddScalarProgram), 3: a[i] * b[i / H]
 * (ExportMulBroadcastLastProgram), 4: a[i] * b[i % H] (ExportMulLeftBroadcastF32XProgram)
 *   src/models/optimized_qwen3_asr/shaders/{pow_scalar_f32,rsqrt_f32,add_scalar,mul_broadcast_last,
 *   mul_left_broadcast_f32x_f32}.py */
int t2c_ew_misc(int op, const void *a, int a_f16, const void *b, int b_f16, void *out, int out_f16, int64_t n, int64_t H,
                float scalar, void *stream);
/* out[r] = mean(x[r, :]) for fp32 x [rows, cols].  Replaces ExportMeanDimProgram
 *   src/models/optimized_qwen3_asr/shaders/mean_dim_f32.py */
int t2c_row_mean_f32(const float *x, float *out, int64_t rows, int64_t cols, void *stream);

/* ------------------------------------------------------------------ tensor parallelism
 * One-shot all-reduce of fp16 tensors over NVLink peer memory (the two
 * per-layer reductions of the row-split o_proj / down_proj partial sums in the
 * tensor-parallel decode step; replaces the NCCL all-reduce a Megatron split
 * would use).  Every rank holds one buffer of t2c_allreduce_buffer_bytes(n_max)
 * bytes (zeroed, 256-byte aligned) mapped into every peer with the IPC helpers;
 * `bufs` lists the tp buffer addresses as seen by this rank (host array),
 * `counter` is this rank's two zeroed device words.  n (a multiple of 8, <= n_max)
 * halves of x are summed in place.  A peer that never arrives: after 1 s the
 * kernel leaves x unreduced and sets T2C_ETIMEOUT in t2c_device_status.
 * The reference runs single-GPU only; there is no counterpart there.
 */
int64_t t2c_allreduce_buffer_bytes(int64_t n_max);
int t2c_ipc_get_handle(const void *ptr, void *handle64, int64_t *offset);
int t2c_ipc_open_handle(const void *handle64, void **ptr);
int t2c_ipc_close_handle(void *ptr);
int t2c_allreduce_sum_f16(void *x, int64_t n, void *const *bufs, int rank, int tp, uint32_t *counter, int64_t n_max,
                          void *stream);

/* Row-parallel quantized linear with the reduction over the tensor-parallel group fused
 * into its epilogue (the o_proj / down_proj of a TP decode step at 1 token):
 *   y = residual + sum over the tp ranks of (x @ W_rank^T)
 * where every rank holds its K-slice W_rank (Q4_K, [N, K / tp] values) and its own copy
 * of residual / y (y may alias residual).  Each 16-row block's fp32 partials are parked
 * are pushed into every rank's buffer (t2c_linear_allreduce_buffer_bytes(n_max) bytes,
 * zeroed, 256-byte aligned, IPC-mapped into every peer like the all-reduce buffer); each
 * CTA then releases a per-launch epoch to every peer once, waits for the peers' CTA of the
 * same index, and sums its rows' partials in rank order: one launch instead of a matvec
 * plus an all-reduce, the same bits on every rank.
 * 1 token, Q4_K, N a multiple of 16 up to 16384 (<= n_max, n_max % 4 == 0), K a multiple of 512, else
 * T2C_EUNSUPPORTED (use t2c_linear + t2c_allreduce_sum_f16).  `counter`: this rank's two
 * zeroed device words (not shared with t2c_allreduce_sum_f16).  A peer that never
 * arrives: after 1 s the block keeps its local partial and T2C_ETIMEOUT is set.
 * The reference runs single-GPU only; there is no counterpart there.
 */
int64_t t2c_linear_allreduce_buffer_bytes(int64_t n_max);
int t2c_linear_allreduce(int wtype, const void *x, const void *w, const void *residual, void *y, int64_t M, int64_t N,
                         int64_t K, void *const *bufs, int rank, int tp, uint32_t *counter, int64_t n_max,
                         void *stream);

#ifdef __cplusplus
}
#endif

#endif /* T2C_SM100_H */

"""CPU restatement of the optimized Qwen3 fp32-activation prefill programs (TEST INFRASTRUCTURE ONLY).

Only ``tests/`` import this module, as the checker of the llama.cpp-style
prefill ops of torch2vk_b200 (kernels.linear_f32, rms_norm_f32,
rms_norm_rope_f32, value_cache_write_f32, fa_mask_opt,
attn_prefill_masked_f32).  Each function restates one reference shader of
``src/models/optimized_qwen3/shaders/`` (paths inside the torch2vk project):

* ``fa_mask_opt``             fa_mask_opt_f16.py (GLSL main: 16 blocks of Br=16 x Bc=64 per word,
                              bit 1 when max <= -FLT_MAX/2, bit 2 when min == max == 0, word
                              stored at row_block * W + word)
* ``rms_norm_rope_token``     rms_norm_rope_token_f32.py (inv_rms over D, norm * w, rotate-half
                              with sign -1 below D/2, cos / sin rows (b * T + t) * D)
* ``rms_norm_mul``            rms_norm_mul_f32.py (x * inversesqrt(sum/H + 1e-6) * w)
* ``value_cache_write``       token_major_value_cache_write_f32_to_f16_pair.py (fp16 of src at row
                              cache_position[t] of each cache; rows past a cache's extent skipped)
* ``flash_attn``              llama_flash_attn_f32_f16_f16.py: softmax(q k^T * scale + mask) v over
                              keys [0, S) with the GQA head map h -> h * NK / NH (fp64 here)
* ``causal_mask``             run.py:258-262 (_prefill_causal_mask)

Pins: the restatements are plain array algebra of the shader bodies; the
classifier is additionally checked against hand-built masks whose codes are
known (tests/test_prefill32_gpu.py).  No reference output vectors exist for
these programs (the reference runs them only on a Vulkan GPU), so parity of
the fp32 arithmetic is checked within the stated tolerances, not bit for bit.
"""

from __future__ import annotations

import numpy as np

FLT_MAX_OVER_2 = np.float32(1.7014117e38)


def causal_mask(chunk_start: int, chunk_length: int, attention_length: int) -> np.ndarray:
    m = np.zeros((chunk_length, attention_length), np.float16)
    for r in range(chunk_length):
        m[r, chunk_start + r + 1:] = np.float16(-np.inf)
    return m


def fa_mask_opt(mask: np.ndarray) -> np.ndarray:
    """uint32 [R, W] codes of an fp16 mask [T, S]."""
    T, S = mask.shape
    W, R = (S + 1023) // 1024, (T + 15) // 16
    out = np.zeros((R, W), np.uint32)
    m = mask.astype(np.float32)
    for rb in range(R):
        for w in range(W):
            word = 0
            for bx in range(16):
                c0 = (w * 16 + bx) * 64
                blk = m[rb * 16:min(T, rb * 16 + 16), c0:min(S, c0 + 64)]
                mn = float(blk.min()) if blk.size else float(FLT_MAX_OVER_2)
                mx = float(blk.max()) if blk.size else -float(FLT_MAX_OVER_2)
                if mx <= -float(FLT_MAX_OVER_2):
                    word |= 1 << (2 * bx)
                if mn == 0.0 and mx == 0.0:
                    word |= 2 << (2 * bx)
            out[rb, w] = word
    return out


def rms_norm_mul(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x64 = x.astype(np.float64)
    inv = 1.0 / np.sqrt((x64 * x64).sum(-1, keepdims=True) / x.shape[-1] + eps)
    return x64 * inv * w.astype(np.float64)


def rms_norm_rope_token(x: np.ndarray, w: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                        eps: float = 1e-6) -> np.ndarray:
    """x [B, T, G, D], w [D], cos / sin [B, T, D] -> [B, T, G, D] (fp64)."""
    D = x.shape[-1]
    n = rms_norm_mul(x, w, eps)
    half = D // 2
    rot = np.concatenate([-n[..., half:], n[..., :half]], axis=-1)
    c = cos.astype(np.float64)[:, :, None, :]
    s = sin.astype(np.float64)[:, :, None, :]
    return n * c + rot * s


def value_cache_write(caches: list[np.ndarray], src: np.ndarray, positions: np.ndarray) -> None:
    """In place: caches [B, S_c, H, D] fp16, src [B, T, H, D] fp32."""
    for t, pos in enumerate(positions.tolist()):
        for c in caches:
            if 0 <= pos < c.shape[1]:
                c[:, pos] = src[:, t].astype(np.float16)


def flash_attn(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray, scale: float) -> np.ndarray:
    """q [B, T, NH, D], k / v [B, S, NK, D], mask [T, S] -> [B, T, NH, D] (fp64)."""
    B, T, NH, D = q.shape
    NK = k.shape[2]
    out = np.zeros((B, T, NH, D))
    m = mask.astype(np.float64)
    for b in range(B):
        for h in range(NH):
            kh = h * NK // NH
            s = q[b, :, h].astype(np.float64) @ k[b, :, kh].astype(np.float64).T * scale + m
            s = s - s.max(-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(-1, keepdims=True)
            out[b, :, h] = p @ v[b, :, kh].astype(np.float64)
    return out

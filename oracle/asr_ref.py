"""fp32 CPU restatement of the Qwen3-ASR audio encoder (TEST INFRASTRUCTURE ONLY).

Only ``tests/`` import this module, as the checker of torch2vk_b200.asr.  It
restates the forward of Qwen3ASRAudioEncoder from the reference's vendored HF
modeling file (paths inside the torch2vk project):

* encoder forward, after the host-side chunking: ``src/qwen_asr/core/transformers_backend/modeling_qwen3_asr.py:752-780``
  (conv2d1..3 + GELU, permute + conv_out, position embedding, gather of the
  valid frames, layers, ln_post, proj1 + GELU, proj2);
* encoder layer: ``:536-576`` (pre-LayerNorm attention and GELU FFN, residuals);
* attention: ``:477-521`` on the eager path (softmax(q k^T * head_dim^-0.5 +
  mask) v, with the block-diagonal additive mask of ``:685-704``).

Pins: ``tests/golden/asr_encoder_tiny.npz`` holds the output of the HF module
itself (imported from the reference tree by ``tests/golden/make_asr_golden.py``)
for seeded parameters and features; ``tests/test_asr_cpu.py`` checks this
restatement against it.  The quantized path's numerics (Q8_0 weights, fp16
activations) are checked on the GPU against this restatement run on the
dequantized weights.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def encoder_forward(params: dict[str, np.ndarray], inputs, cfg) -> np.ndarray:
    """[tokens, output_dim] fp32 for the prepared inputs (torch2vk_b200.asr.AsrInputs)."""
    P = {k: torch.from_numpy(np.asarray(v, dtype=np.float32)) for k, v in params.items()}
    with torch.no_grad():
        x = torch.from_numpy(inputs.padded_feature)
        for i in (1, 2, 3):
            x = F.gelu(F.conv2d(x, P[f"conv2d{i}.weight"], P[f"conv2d{i}.bias"], stride=2, padding=1))
        b, c, f, t = x.shape
        x = x.permute(0, 3, 1, 2).reshape(b, t, c * f) @ P["conv_out.weight"].T
        x = x + torch.from_numpy(inputs.position_embedding)
        h = x.reshape(b * t, -1)[torch.from_numpy(inputs.compact_index)]
        mask = torch.from_numpy(inputs.attention_mask)[0, 0]
        n, d = h.shape
        H, hd = cfg.heads, d // cfg.heads
        for i in range(cfg.layers):
            p = f"layers.{i}."
            r = h
            a = F.layer_norm(h, (d,), P[p + "self_attn_layer_norm.weight"], P[p + "self_attn_layer_norm.bias"], cfg.eps)
            q = (a @ P[p + "self_attn.q_proj.weight"].T + P[p + "self_attn.q_proj.bias"]).view(n, H, hd).transpose(0, 1)
            k = (a @ P[p + "self_attn.k_proj.weight"].T + P[p + "self_attn.k_proj.bias"]).view(n, H, hd).transpose(0, 1)
            v = (a @ P[p + "self_attn.v_proj.weight"].T + P[p + "self_attn.v_proj.bias"]).view(n, H, hd).transpose(0, 1)
            s = q @ k.transpose(1, 2) * hd ** -0.5 + mask
            o = (torch.softmax(s, dim=-1) @ v).transpose(0, 1).reshape(n, d)
            h = r + o @ P[p + "self_attn.out_proj.weight"].T + P[p + "self_attn.out_proj.bias"]
            r = h
            a = F.layer_norm(h, (d,), P[p + "final_layer_norm.weight"], P[p + "final_layer_norm.bias"], cfg.eps)
            a = F.gelu(a @ P[p + "fc1.weight"].T + P[p + "fc1.bias"])
            h = r + a @ P[p + "fc2.weight"].T + P[p + "fc2.bias"]
        h = F.layer_norm(h, (d,), P["ln_post.weight"], P["ln_post.bias"], cfg.eps)
        h = F.gelu(h @ P["proj1.weight"].T + P["proj1.bias"])
        out = h @ P["proj2.weight"].T + P["proj2.bias"]
    return out.numpy()


def q8_rows(w: np.ndarray) -> np.ndarray:
    """[rows, K] view of a weight (conv: k = (ic, fh, fw), as conv2d_q8_0w_f32b_f16.py:128), zero-padded
    to whole 32-value Q8_0 blocks."""
    m = w.reshape(w.shape[0], -1)
    kp = (m.shape[1] + 31) // 32 * 32
    if kp != m.shape[1]:
        m = np.concatenate([m, np.zeros((m.shape[0], kp - m.shape[1]), dtype=m.dtype)], axis=1)
    return np.ascontiguousarray(m, dtype=np.float32)


def dequantized_params(params: dict[str, np.ndarray], names, quantize, dequantize) -> dict[str, np.ndarray]:
    """params with every tensor in ``names`` replaced by its Q8_0 round trip (same shape)."""
    out = dict(params)
    for n in names:
        w = params[n]
        rows = q8_rows(w)
        deq = dequantize(quantize(rows, "q8_0"), "q8_0", rows.shape[1])
        k = int(np.prod(w.shape[1:]))
        out[n] = deq[:, :k].reshape(w.shape).astype(np.float32)
    return out

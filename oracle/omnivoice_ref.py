"""Reference path for the OmniVoice LLM forward (TEST INFRASTRUCTURE ONLY).

The OmniVoice model (src/omnivoice/models/omnivoice.py) is a Qwen3 decoder
called with inputs_embeds and a 4-D additive attention mask: the embeddings
are text rows, or the sum over the codebooks of audio rows
(_prepare_embed_inputs, omnivoice.py:360-380), and the audio heads are a
plain linear over the final-normed hidden states (omnivoice.py:224-228).  The
quantized program (quantized_omnivoice/dispatch/llm_forward.py) computes the
same graph on dequantized GGUF blocks.

This oracle is the HF transformers Qwen3 stack (fp32, CPU, eager attention)
built by oracle/qwen3_ref.build (Q4_K_M linears dequantized back into the HF
modules) and driven layer by layer with the explicit mask; the Q8_0 text and
audio embeddings and the Q6_K audio heads are quantized by the C oracle and
dequantized for the fp32 computation.  The input embedding follows the
quantized shader (custom_shaders.py:150-181): fp32 sum in codebook order,
rounded to fp16.

Only tests/ import this module.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from oracle import oracle as O
from oracle import qwen3_ref


@dataclass
class OmniPacked:
    pm: qwen3_ref.PackedModel
    text_q8: np.ndarray
    audio_q8: np.ndarray
    heads_q6: np.ndarray
    text_deq: np.ndarray
    audio_deq: np.ndarray
    heads_deq: np.ndarray
    codebooks: int
    audio_vocab: int


def build(hidden: int, layers: int, heads: int, kv_heads: int, head_dim: int, intermediate: int, text_vocab: int,
          *, codebooks: int = 8, audio_vocab: int = 1025, seed: int = 0) -> OmniPacked:
    pm = qwen3_ref.build(hidden, layers, heads, kv_heads, head_dim, intermediate, text_vocab, seed=seed,
                         topology="q4_k_m")
    rng = np.random.default_rng(seed + 1)
    text = pm.hf.model.embed_tokens.weight.detach().numpy().astype(np.float32)
    audio = (rng.standard_normal((codebooks * audio_vocab, hidden)) * 0.02).astype(np.float32)
    heads_w = (rng.standard_normal((codebooks * audio_vocab, hidden)) * 0.02).astype(np.float32)
    text_q8 = O.quantize(text, "q8_0")
    audio_q8 = O.quantize(audio, "q8_0")
    heads_q6 = O.quantize(heads_w, "q6_k")
    return OmniPacked(pm, text_q8, audio_q8, heads_q6, O.dequantize_np(text_q8, "q8_0", hidden),
                      O.dequantize_np(audio_q8, "q8_0", hidden), O.dequantize_np(heads_q6, "q6_k", hidden),
                      codebooks, audio_vocab)


def input_embeds(om: OmniPacked, ids: np.ndarray, audio_mask: np.ndarray) -> np.ndarray:
    """fp16 [B, S, H]: text row ids[b, 0, s], or the fp32 codebook-order sum of audio rows."""
    B, C, S = ids.shape
    out = np.empty((B, S, om.text_deq.shape[1]), np.float16)
    for b in range(B):
        for s in range(S):
            if audio_mask[b, s]:
                acc = np.zeros(om.audio_deq.shape[1], np.float32)
                for c in range(C):
                    acc = (acc + om.audio_deq[c * om.audio_vocab + ids[b, c, s]]).astype(np.float32)
                out[b, s] = acc.astype(np.float16)
            else:
                out[b, s] = om.text_deq[ids[b, 0, s]].astype(np.float16)
    return out


@torch.no_grad()
def llm_forward(om: OmniPacked, embeds: np.ndarray, mask: np.ndarray) -> tuple[list[torch.Tensor], torch.Tensor]:
    """Per-layer outputs [B, S, H] and the audio-head logits [B, S, C * V] (fp32) of the HF Qwen3 layers
    run on embeds (fp16 values) under the additive mask [B, 1, S, S] (-inf entries become -FLT_MAX, as the
    reference's host mask is before its fp16 conversion)."""
    hf = om.pm.hf
    hf.config._attn_implementation = "eager"
    x = torch.from_numpy(embeds.astype(np.float32))
    B, S, _ = x.shape
    m = torch.from_numpy(np.maximum(mask.astype(np.float32), np.finfo(np.float32).min))
    pos = torch.arange(S)[None].expand(B, -1)
    pe = hf.model.rotary_emb(x, pos)
    outs = []
    for layer in hf.model.layers:
        x = layer(x, attention_mask=m, position_ids=pos, position_embeddings=pe)
        x = x[0] if isinstance(x, tuple) else x
        outs.append(x.clone())
    normed = hf.model.norm(x)
    return outs, normed @ torch.from_numpy(om.heads_deq).T

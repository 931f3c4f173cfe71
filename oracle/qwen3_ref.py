"""Reference PyTorch path for Qwen3 parity (TEST INFRASTRUCTURE ONLY).

"The reference's PyTorch dequantize-then-compute path": the HF transformers
Qwen3ForCausalLM (third-party; the reference exports this class at
src/models/quantized_qwen3/export.py:16,102-119) run in fp32 on the CPU with
its linear weights replaced by the dequantized GGUF blocks the GPU consumes.

Recipe (seeded, deterministic):
  * torch.manual_seed(seed); Qwen3ForCausalLM(config) -> HF default init
    (N(0, 0.02) linears/embeddings, RMSNorm weights 1.0);
  * every linear is quantized by the CPU oracle (gguf_quant_ref.c) with the
    requested topology (pure Q4_K, or Q4_K_M: Q6_K v_proj/down_proj in the
    more-bits layers, src/torch2vk/quantize/gguf.py:150-161);
  * embeddings are stored F16 (the GGUF f16_tensor_names mechanism,
    quantize/gguf.py:36,49-52), the tied LM head as Q6_K of the embedding
    matrix (models/quantized_qwen3/quantization.py:17-23);
  * the HF model gets the dequantized weights back and computes in fp32.

Only tests/ and bench.py's CPU-baseline leg import this module.
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass

import numpy as np
import torch

from oracle import oracle as O


@dataclass
class PackedModel:
    """Packed GGUF tensors (numpy uint8 rows) plus the matching fp32 HF model."""

    hf: torch.nn.Module
    cfg: object
    packed: dict[str, tuple[np.ndarray, str]]  # name -> (bytes [rows, row_bytes], kind)
    embed_f16: np.ndarray
    norms: dict[str, np.ndarray]


def hf_config(hidden: int, layers: int, heads: int, kv_heads: int, head_dim: int, intermediate: int, vocab: int,
              eps: float = 1e-6, theta: float = 1e6):
    from transformers import Qwen3Config

    return Qwen3Config(hidden_size=hidden, intermediate_size=intermediate, num_hidden_layers=layers,
                       num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=head_dim, vocab_size=vocab,
                       rms_norm_eps=eps, rope_theta=theta, tie_word_embeddings=False, max_position_embeddings=40960,
                       attention_bias=False, torch_dtype="float32")


def build(hidden: int, layers: int, heads: int, kv_heads: int, head_dim: int, intermediate: int, vocab: int, *,
          seed: int = 0, topology: str = "q4_k_m", lm_head_kind: str = "q6_k") -> PackedModel:
    from transformers import Qwen3ForCausalLM

    torch.manual_seed(seed)
    cfg = hf_config(hidden, layers, heads, kv_heads, head_dim, intermediate, vocab)
    hf = Qwen3ForCausalLM(cfg).float().eval()
    q6 = set(O.q4_k_m_more_bits_layer_indices(layers)) if topology == "q4_k_m" else set()
    packed: dict[str, tuple[np.ndarray, str]] = {}
    with torch.no_grad():
        embed = hf.model.embed_tokens.weight.detach().numpy().astype(np.float32)
        embed_f16 = embed.astype(np.float16)
        hf.model.embed_tokens.weight.copy_(torch.from_numpy(embed_f16.astype(np.float32)))
        head_bytes = O.quantize(embed, lm_head_kind)
        packed["lm_head.weight"] = (head_bytes, lm_head_kind)
        hf.lm_head.weight.copy_(torch.from_numpy(O.dequantize_np(head_bytes, lm_head_kind, hidden)))
        for i, layer in enumerate(hf.model.layers):
            mods = {
                "self_attn.q_proj": layer.self_attn.q_proj,
                "self_attn.k_proj": layer.self_attn.k_proj,
                "self_attn.v_proj": layer.self_attn.v_proj,
                "self_attn.o_proj": layer.self_attn.o_proj,
                "mlp.gate_proj": layer.mlp.gate_proj,
                "mlp.up_proj": layer.mlp.up_proj,
                "mlp.down_proj": layer.mlp.down_proj,
            }
            for name, mod in mods.items():
                kind = "q6_k" if (i in q6 and name in ("self_attn.v_proj", "mlp.down_proj")) else "q4_k"
                w = mod.weight.detach().numpy().astype(np.float32)
                blob = O.quantize(w, kind)
                packed[f"model.layers.{i}.{name}.weight"] = (blob, kind)
                mod.weight.copy_(torch.from_numpy(O.dequantize_np(blob, kind, w.shape[1])))
    norms = {n: p.detach().numpy().astype(np.float32).copy() for n, p in hf.named_parameters() if p.dim() == 1}
    return PackedModel(hf=hf, cfg=cfg, packed=packed, embed_f16=embed_f16, norms=norms)


def prompt_ids(tokens: int, vocab: int, seed: int = 0, batch: int = 1) -> torch.Tensor:
    """Uniform random prompt ids (torch.Generator().manual_seed(seed))."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (batch, tokens), generator=gen, dtype=torch.int64)


@torch.no_grad()
def prefill_hidden(hf: torch.nn.Module, ids: torch.Tensor) -> tuple[list[torch.Tensor], torch.Tensor]:
    """Per-layer residual-stream outputs and the last-position logits of the fp32 model."""
    out = hf(input_ids=ids, output_hidden_states=True, use_cache=False)
    hs = list(out.hidden_states[1:])  # after each layer (the last one is after the final norm)
    return hs, out.logits[:, -1, :]


@torch.no_grad()
def greedy(hf: torch.nn.Module, ids: torch.Tensor, steps: int) -> tuple[torch.Tensor, list[float]]:
    """Greedy tokens [batch, steps] and, per step, the top-1 minus top-2 logit gap."""
    out = hf(input_ids=ids, use_cache=True)
    past = out.past_key_values
    logits = out.logits[:, -1, :]
    tokens, gaps = [], []
    for _ in range(steps):
        top = torch.topk(logits, 2, dim=-1)
        gaps.append(float((top.values[:, 0] - top.values[:, 1]).min()))
        nxt = top.indices[:, :1]
        tokens.append(nxt)
        out = hf(input_ids=nxt, past_key_values=past, use_cache=True)
        past = out.past_key_values
        logits = out.logits[:, -1, :]
    return torch.cat(tokens, dim=1), gaps


@torch.no_grad()
def time_decode_cpu(hf: torch.nn.Module, ids: torch.Tensor, steps: int, threads: int | None = None) -> dict:
    """CPU baseline: fp32 HF decode tok/s on the host cores (prefill excluded from the timing)."""
    threads = threads or (os.cpu_count() or 1)
    torch.set_num_threads(threads)
    out = hf(input_ids=ids, use_cache=True)
    past = out.past_key_values
    nxt = out.logits[:, -1:, :].argmax(-1)
    t0 = time.perf_counter()
    for _ in range(steps):
        out = hf(input_ids=nxt, past_key_values=past, use_cache=True)
        past = out.past_key_values
        nxt = out.logits[:, -1:, :].argmax(-1)
    dt = time.perf_counter() - t0
    return {"tok_s": ids.shape[0] * steps / dt, "seconds": dt, "threads": threads, "steps": steps}

"""Qwen3-ASR end to end: mel -> audio encoder -> audio rows injected into the
prompt -> text decoder prefill -> 64 greedy tokens, for a batch of two clips.

The encoder is the benched tower (d_model 896, 480-channel convolutions) with
two layers, Q8_0 weights; its output rows are checked against the oracle
encoder (oracle/asr_ref.py, pinned to the reference's HF module) on the same
dequantized weights.  The text decoder (Qwen3-0.6B widths, two layers, vocab
trimmed to 8192, Q4_K_M) is checked against the oracle HF model fed the same
audio rows as inputs_embeds: the 64 greedy token ids of every clip must be
identical.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from test_qwen3_gpu import upload

pytestmark = pytest.mark.gpu

STEPS = 64


@torch.no_grad()
def _oracle_greedy(hf, embeds: torch.Tensor, steps: int) -> torch.Tensor:
    out = hf(inputs_embeds=embeds, use_cache=True)
    past, logits = out.past_key_values, out.logits[:, -1, :]
    toks = []
    for _ in range(steps):
        nxt = logits.argmax(-1, keepdim=True)
        toks.append(nxt)
        out = hf(input_ids=nxt, past_key_values=past, use_cache=True)
        past, logits = out.past_key_values, out.logits[:, -1, :]
    return torch.cat(toks, dim=1)


def test_asr_pipeline_tokens_match_oracle(oracle):
    from oracle import asr_ref, qwen3_ref
    from torch2vk_b200.asr import AsrEncoderConfig, prepare_inputs, quantized_names, random_params
    from torch2vk_b200.asr_pipeline import AsrPipeline
    from torch2vk_b200.qwen3 import Qwen3Config

    enc_cfg = dataclasses.replace(AsrEncoderConfig.qwen3_asr_0_6b(), layers=2)
    enc_params = random_params(enc_cfg, seed=0)
    text_cfg = Qwen3Config(hidden=1024, layers=2, heads=16, kv_heads=8, head_dim=128, intermediate=3072, vocab=8192)
    pm = qwen3_ref.build(text_cfg.hidden, text_cfg.layers, text_cfg.heads, text_cfg.kv_heads, text_cfg.head_dim,
                         text_cfg.intermediate, text_cfg.vocab, seed=0, topology="q4_k_m")
    batch, frames = 2, 3000
    pipe = AsrPipeline(enc_cfg, enc_params, text_cfg, upload(pm, text_cfg), batch=batch, frames=frames, prefix=9,
                       suffix=6, max_new_tokens=STEPS)
    rng = np.random.default_rng(4)
    mels = [rng.standard_normal((enc_cfg.num_mel_bins, frames)).astype(np.float32) for _ in range(batch)]
    gen = torch.Generator().manual_seed(1)
    prefix = torch.randint(0, text_cfg.vocab, (1, 9), generator=gen)
    suffix = torch.randint(0, text_cfg.vocab, (1, 6), generator=gen)
    ids = pipe.prompt(prefix, suffix, placeholder=7)
    got = pipe.transcribe(pipe.upload(mels), ids).cpu()
    feats = pipe.features.float().cpu()

    deq = asr_ref.dequantized_params(enc_params, quantized_names(enc_cfg), oracle.quantize, oracle.dequantize)
    for b in range(batch):
        ref = asr_ref.encoder_forward(deq, prepare_inputs(mels[b], enc_cfg), enc_cfg)
        f = feats[b].numpy()
        cos = float((f * ref).sum() / (np.linalg.norm(f) * np.linalg.norm(ref)))
        assert cos >= 0.999 and float(np.abs(f - ref).max()) <= 2e-2 * float(np.abs(ref).max()), (b, cos)

    embeds = pm.hf.model.embed_tokens(ids.cpu()).clone()
    embeds[:, 9:9 + pipe.audio_tokens, :] = feats
    ref_tokens = _oracle_greedy(pm.hf, embeds, STEPS)
    assert torch.equal(got, ref_tokens), f"got {got.tolist()}\nref {ref_tokens.tolist()}"
    from torch2vk_b200 import kernels

    assert kernels.device_status() == 0

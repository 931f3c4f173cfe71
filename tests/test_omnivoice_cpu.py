"""OmniVoice host logic and the oracle's pin (CPU only).

The oracle drives HF Qwen3 decoder layers one by one with an explicit mask;
with a causal mask that must reproduce HF's own Qwen3Model forward on the
same inputs_embeds, which pins the layer driving (rotary embeddings,
positions, mask convention).  Its input embedding must agree with the
model-level formula (omnivoice.py:360-380: where(audio_mask, sum of shifted
audio rows, text rows)) up to the order of the fp32 sum.
"""

from __future__ import annotations

import numpy as np
import torch


def _cfg():
    from torch2vk_b200.omnivoice import OmniVoiceConfig
    from torch2vk_b200.qwen3 import Qwen3Config

    return OmniVoiceConfig(llm=Qwen3Config(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, intermediate=512,
                                           vocab=300), codebooks=3, audio_vocab=17, audio_mask_id=16)


def test_prepare_inputs_layout():
    """The CFG pair's ids, audio mask and attention mask (input_prep.py:76-115 with given token ids)."""
    from torch2vk_b200.omnivoice import prepare_inputs

    cfg = _cfg()
    inp = prepare_inputs(np.array([5, 6]), np.array([7, 8, 9]), 4, cfg)
    assert inp.input_ids.shape == (2, 3, 9) and inp.cond_audio_start == 5
    assert (inp.input_ids[0, :, :5] == [5, 6, 7, 8, 9]).all() and (inp.input_ids[0, :, 5:] == 16).all()
    assert (inp.input_ids[1] == 16).all()
    assert inp.audio_mask.tolist() == [[0] * 5 + [1] * 4, [1] * 4 + [0] * 5]
    m = inp.attention_mask
    assert m.dtype == np.float16 and (m[0] == 0).all()
    vis = m[1, 0] == 0
    assert vis[:4, :4].all() and not vis[:4, 4:].any() and not vis[4:, :4].any()
    assert (vis[4:, 4:] == np.eye(5, dtype=bool)).all()
    assert np.isneginf(m[1, 0, 0, 5])


def _om():
    from oracle import omnivoice_ref

    c = _cfg()
    return c, omnivoice_ref.build(c.llm.hidden, c.llm.layers, c.llm.heads, c.llm.kv_heads, c.llm.head_dim,
                                  c.llm.intermediate, c.llm.vocab, codebooks=c.codebooks,
                                  audio_vocab=c.audio_vocab)


def test_oracle_layer_driving_matches_hf_model_forward():
    from oracle import omnivoice_ref

    c, om = _om()
    S = 11
    rng = np.random.default_rng(0)
    embeds = (rng.standard_normal((2, S, c.llm.hidden)) * 0.5).astype(np.float16)
    causal = np.triu(np.full((S, S), -np.inf, np.float32), 1).astype(np.float16)
    outs, _ = omnivoice_ref.llm_forward(om, embeds, np.broadcast_to(causal, (2, 1, S, S)).copy())
    with torch.no_grad():
        ref = om.pm.hf.model(inputs_embeds=torch.from_numpy(embeds.astype(np.float32)), output_hidden_states=True)
    for got, want in zip(outs[:-1], ref.hidden_states[1:-1]):
        assert torch.allclose(got, want, atol=1e-5, rtol=1e-5)


def test_oracle_input_embeds_match_model_formula():
    from oracle import omnivoice_ref
    from torch2vk_b200.omnivoice import prepare_inputs

    c, om = _om()
    rng = np.random.default_rng(1)
    inp = prepare_inputs(rng.integers(0, c.llm.vocab, 3), rng.integers(0, c.llm.vocab, 4), 6, c)
    ids = inp.input_ids.copy()
    ids[0, :, 7:9] = rng.integers(0, 16, (c.codebooks, 2))
    got = omnivoice_ref.input_embeds(om, ids, inp.audio_mask)
    t = torch.from_numpy(ids)
    text = torch.from_numpy(om.text_deq)[t[:, 0, :]]
    am = torch.from_numpy(inp.audio_mask.astype(bool))
    shifted = t * am.unsqueeze(1) + (torch.arange(c.codebooks) * c.audio_vocab)[None, :, None]
    audio = torch.from_numpy(om.audio_deq)[shifted].sum(dim=1)
    want = torch.where(am.unsqueeze(-1), audio, text).numpy()
    assert np.allclose(got.astype(np.float32), want, rtol=2e-3, atol=1e-6)

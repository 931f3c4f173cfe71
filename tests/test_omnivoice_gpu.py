"""OmniVoice LLM forward (the per-step program of quantized_omnivoice/dispatch/llm_forward.py) against the
oracle (oracle/omnivoice_ref.py: HF Qwen3 layers in fp32 on the dequantized blocks, explicit 4-D mask).

Gates: the input embedding bit for bit (fp32 codebook-order sums rounded to
fp16); every layer output within max-abs 2e-2 and cosine >= 0.999 of the
oracle's (the Qwen3 decoder gates); the audio-head logits with cosine >= 0.999
and max |err| <= 2e-2 * max |ref|; the graph-replayed step equal to the direct
one.  Shapes: OmniVoice's LLM widths (hidden 1024, 16 Q / 8 KV heads, FFN
3072), three layers, the text vocabulary trimmed to 4096, the real audio heads
(8 codebooks x 1025), the CFG batch of two over 150 positions.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from test_qwen3_gpu import _check_layer

pytestmark = pytest.mark.gpu


def _setup(layers=3, text_vocab=4096, target_len=100):
    from oracle import omnivoice_ref
    from test_qwen3_gpu import upload
    from torch2vk_b200.omnivoice import OmniVoiceConfig, OmniVoiceLLM, OmniVoiceWeights, prepare_inputs
    from torch2vk_b200.qwen3 import QWeight, Qwen3Config

    llm = Qwen3Config(hidden=1024, layers=layers, heads=16, kv_heads=8, head_dim=128, intermediate=3072,
                      vocab=text_vocab)
    cfg = OmniVoiceConfig(llm=llm)
    om = omnivoice_ref.build(llm.hidden, llm.layers, llm.heads, llm.kv_heads, llm.head_dim, llm.intermediate,
                             llm.vocab, codebooks=cfg.codebooks, audio_vocab=cfg.audio_vocab)
    qw = upload(om.pm, llm)
    w = OmniVoiceWeights(text_embed=torch.from_numpy(om.text_q8).cuda(),
                         audio_embed=torch.from_numpy(om.audio_q8).cuda(), layers=qw.layers,
                         final_norm=qw.final_norm, audio_heads=QWeight(torch.from_numpy(om.heads_q6).cuda(), "q6_k"))
    rng = np.random.default_rng(3)
    inputs = prepare_inputs(rng.integers(0, text_vocab, 14), rng.integers(0, text_vocab, 36), target_len, cfg)
    # a decoding step part-way through: some target positions already hold audio ids
    ids = inputs.input_ids.copy()
    start = inputs.cond_audio_start
    known = rng.random(target_len) < 0.4
    codes = rng.integers(0, cfg.audio_vocab - 1, (cfg.codebooks, target_len))
    ids[0, :, start:][:, known] = codes[:, known]
    ids[1, :, :target_len][:, known] = codes[:, known]
    inputs = type(inputs)(ids, inputs.audio_mask, inputs.attention_mask, inputs.target_len, start)
    runner = OmniVoiceLLM(cfg, w, batch=2, seq=ids.shape[2])
    return cfg, om, inputs, runner


def test_omnivoice_input_embed_is_exact():
    from oracle import omnivoice_ref
    from torch2vk_b200 import kernels

    cfg, om, inputs, runner = _setup(layers=1)
    runner.upload(inputs)
    kernels.device_status(clear=True)
    runner._embed()
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    want = omnivoice_ref.input_embeds(om, inputs.input_ids, inputs.audio_mask)
    got = runner.h.view(want.shape).cpu().numpy()
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


def test_omnivoice_llm_forward_matches_oracle():
    from oracle import omnivoice_ref
    from torch2vk_b200 import kernels

    cfg, om, inputs, runner = _setup()
    runner.upload(inputs)
    outs: list[torch.Tensor] = []
    logits = runner.forward_device(layer_outputs=outs).float().cpu()
    embeds = omnivoice_ref.input_embeds(om, inputs.input_ids, inputs.audio_mask)
    ref_outs, ref_logits = omnivoice_ref.llm_forward(om, embeds, inputs.attention_mask)
    for i, (g, r) in enumerate(zip(outs, ref_outs)):
        _check_layer(g, r.reshape(g.shape), f"OmniVoice layer {i}")
    g, r = logits.flatten(), ref_logits.flatten()
    cos = float(torch.nn.functional.cosine_similarity(g, r, dim=0))
    assert cos >= 0.999 and float((g - r).abs().max()) <= 2e-2 * float(r.abs().max()), cos
    # graph replay of the same step gives the same logits
    replay = runner.forward(inputs).float().cpu()
    assert torch.equal(replay, logits)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("layout", ["head_major", "token_major"])
def test_attn_masked_gqa_matches_fp32(layout):
    """Bidirectional GQA attention under a per-sequence additive mask (the OmniVoice CFG pair's masks, -inf
    entries) against fp32 torch: |err| <= 4e-3 |ref| + 2e-3."""
    from torch2vk_b200 import kernels
    from torch2vk_b200.omnivoice import OmniVoiceConfig, prepare_inputs

    torch.manual_seed(0)
    B, NH, NK, D = 2, 16, 8, 128
    cfg = OmniVoiceConfig.omnivoice()
    inp = prepare_inputs(np.arange(20), np.arange(40), 90, cfg)
    T = inp.input_ids.shape[2]
    mask = torch.from_numpy(inp.attention_mask).cuda()
    q = torch.randn(B, NH, T, D, device="cuda").half()
    k = torch.randn(B, NK, T, D, device="cuda").half()
    v = torch.randn(B, NK, T, D, device="cuda").half()
    kk, vv = k.float().repeat_interleave(NH // NK, 1), v.float().repeat_interleave(NH // NK, 1)
    ref = torch.softmax(q.float() @ kk.transpose(-1, -2) / D ** 0.5 + mask.float(), -1) @ vv
    if layout == "head_major":
        out = kernels.attn_masked_gqa(q, k, v, mask, batch=B, tokens=T, n_heads=NH, n_kv=NK, head_dim=D,
                                      layout="head_major")
    else:
        out = kernels.attn_masked_gqa(q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous(),
                                      v.transpose(1, 2).contiguous(), mask, batch=B, tokens=T, n_heads=NH, n_kv=NK,
                                      head_dim=D).transpose(1, 2)
    err = (out.float() - ref).abs()
    assert bool((err <= 4e-3 * ref.abs() + 2e-3).all()), float(err.max())

"""Qwen3-ASR audio encoder, CPU side: host input preparation and the fp32 oracle, pinned against the
output of the reference's HF module (tests/golden/asr_encoder_tiny.npz, made by make_asr_golden.py)."""

from pathlib import Path

import numpy as np

from oracle import asr_ref
from torch2vk_b200.asr import AsrEncoderConfig, feat_extract_output_lengths, prepare_inputs, random_params

GOLDEN = Path(__file__).resolve().parent / "golden" / "asr_encoder_tiny.npz"
TINY = AsrEncoderConfig(num_mel_bins=128, d_model=128, layers=2, heads=2, ffn=256, output_dim=96, conv_channels=32,
                        n_window=50, n_window_infer=200)


def _golden():
    g = np.load(GOLDEN)
    mel = np.random.default_rng(int(g["mel_seed"])).standard_normal((TINY.num_mel_bins, int(g["frames"])))
    return g, mel.astype(np.float32), random_params(TINY, seed=int(g["param_seed"]))


def test_feat_extract_output_lengths():
    # 3000 mel frames = 30 chunks of 100 -> 13 tokens each (the 0.6B model's 390 audio tokens)
    assert int(feat_extract_output_lengths(np.array([3000]))[0]) == 390
    for n in (1, 50, 99, 100, 101, 250, 777):
        chunks = [100] * (n // 100) + ([n % 100] if n % 100 else [])
        per_chunk = 0
        for c in chunks:
            t = c
            for _ in range(3):
                t = (t + 2 - 3) // 2 + 1
            per_chunk += t
        assert int(feat_extract_output_lengths(np.array([n]))[0]) == per_chunk


def test_prepare_inputs_matches_golden():
    g, mel, _ = _golden()
    inp = prepare_inputs(mel, TINY)
    assert np.array_equal(inp.cu_seqlens, g["cu_seqlens"])
    assert np.array_equal(inp.compact_index, g["compact_index"])
    n = inp.compact_index.shape[0]
    assert inp.attention_mask.shape == (1, 1, n, n)
    # block-diagonal windows: zero inside, the most negative float outside
    a, b = int(g["cu_seqlens"][1]), int(g["cu_seqlens"][2])
    assert inp.attention_mask[0, 0, a, a] == 0 and inp.attention_mask[0, 0, 0, a] < -1e38


def test_oracle_matches_reference_module():
    g, mel, params = _golden()
    out = asr_ref.encoder_forward(params, prepare_inputs(mel, TINY), TINY)
    golden = g["golden"]
    assert out.shape == golden.shape
    assert float(np.abs(out - golden).max()) <= 1e-4 * (1 + float(np.abs(golden).max()))

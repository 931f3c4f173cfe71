"""Golden output of the reference's Qwen3-ASR audio encoder for seeded parameters and features.

Run in a container that has the torch2vk source tree (it imports the vendored HF modeling file
src/qwen_asr/core/transformers_backend/modeling_qwen3_asr.py directly, because the package's
__init__ needs `nagisa`, which is absent):

    python tests/golden/make_asr_golden.py /path/to/torch2vk

The exported encoder attends within block-diagonal windows (cu_seqlens; the reference passes
them to its sdpa_masked shader as an additive mask, pytorch_modules.py:92-106).  The HF module
does that on its flash-attention (varlen) path only; its eager forward calls the layers without a
mask.  This script therefore runs the HF module with every layer given the module's own window
mask (Qwen3ASRAudioEncoder._prepare_attention_mask, modeling_qwen3_asr.py:685-704).

Writes tests/golden/asr_encoder_tiny.npz: the encoder configuration, the seeds, the host-side
window boundaries and gather index, and the HF module's fp32 output.  Parameters and features are
regenerated from the seeds by torch2vk_b200.asr.random_params / numpy's generator.  Before writing,
the script checks that oracle/asr_ref.py reproduces the HF output.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle import asr_ref  # noqa: E402
from torch2vk_b200.asr import AsrEncoderConfig, prepare_inputs, random_params  # noqa: E402

TINY = AsrEncoderConfig(num_mel_bins=128, d_model=128, layers=2, heads=2, ffn=256, output_dim=96, conv_channels=32,
                        n_window=50, n_window_infer=200)
PARAM_SEED, MEL_SEED, FRAMES = 11, 4, 250


def tiny_mel() -> np.ndarray:
    return np.random.default_rng(MEL_SEED).standard_normal((TINY.num_mel_bins, FRAMES)).astype(np.float32)


def load_hf(reference_root: Path):
    base = reference_root / "src" / "qwen_asr" / "core" / "transformers_backend"
    pkg = types.ModuleType("qwen_asr_tb")
    pkg.__path__ = [str(base)]
    sys.modules["qwen_asr_tb"] = pkg
    mods = {}
    for name in ("configuration_qwen3_asr", "modeling_qwen3_asr"):
        spec = importlib.util.spec_from_file_location(f"qwen_asr_tb.{name}", base / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[f"qwen_asr_tb.{name}"] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods["configuration_qwen3_asr"], mods["modeling_qwen3_asr"]


def main() -> None:
    reference_root = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(os.environ["T2C_REFERENCE_ROOT"])
    conf_mod, model_mod = load_hf(reference_root)
    c = TINY
    hf_cfg = conf_mod.Qwen3ASRAudioEncoderConfig(
        num_mel_bins=c.num_mel_bins, encoder_layers=c.layers, encoder_attention_heads=c.heads, encoder_ffn_dim=c.ffn,
        d_model=c.d_model, output_dim=c.output_dim, n_window=c.n_window, n_window_infer=c.n_window_infer,
        downsample_hidden_size=c.conv_channels, max_source_positions=c.max_source_positions)
    hf_cfg._attn_implementation = "eager"
    model = model_mod.Qwen3ASRAudioEncoder(hf_cfg).eval()
    layer_forward = model_mod.Qwen3ASRAudioEncoderLayer.forward

    def windowed_forward(self, hidden_states, cu_seqlens, attention_mask=None, **kwargs):
        if attention_mask is None:
            attention_mask = model._prepare_attention_mask(hidden_states, cu_seqlens)
        return layer_forward(self, hidden_states, cu_seqlens, attention_mask=attention_mask, **kwargs)

    model_mod.Qwen3ASRAudioEncoderLayer.forward = windowed_forward
    params = random_params(c, seed=PARAM_SEED)
    state = {k: torch.from_numpy(v) for k, v in params.items()}
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not unexpected and all("positional_embedding" in m for m in missing), (missing, unexpected)
    mel = tiny_mel()
    with torch.no_grad():
        out = model(input_features=torch.from_numpy(mel), feature_lens=torch.tensor([FRAMES])).last_hidden_state
    golden = out.numpy().astype(np.float32)
    inputs = prepare_inputs(mel, c)
    mine = asr_ref.encoder_forward(params, inputs, c)
    err = float(np.abs(mine - golden).max())
    assert err <= 1e-4 * (1 + float(np.abs(golden).max())), f"oracle vs HF: max err {err}"
    np.savez_compressed(
        Path(__file__).resolve().parent / "asr_encoder_tiny.npz",
        param_seed=PARAM_SEED, mel_seed=MEL_SEED, frames=FRAMES, golden=golden, cu_seqlens=inputs.cu_seqlens,
        compact_index=inputs.compact_index)
    print(f"wrote asr_encoder_tiny.npz: tokens {golden.shape[0]}, windows {np.diff(inputs.cu_seqlens).tolist()}, "
          f"oracle max err {err:.2e}")


if __name__ == "__main__":
    main()

"""Qwen3-ASR audio encoder on the sm_100a kernels (configuration 5 of the hot path).

The reference exports the audio tower of Qwen3-ASR-0.6B with Q8_0 weights and
fp16 activations (src/models/quantized_qwen3_asr/dispatch/audio_encoder.py) and
prepares its inputs on the host (src/models/quantized_qwen3_asr/pytorch_modules.py:50-110):
the log-mel features are cut into 100-frame chunks (n_window = 50), each chunk
goes through three 3x3 stride-2 convolutions with GELU, a bias-free linear
(conv_out) and a sinusoidal position embedding; the valid frames of all chunks
are gathered into one token sequence, which runs through the encoder layers
with block-diagonal attention windows (n_window_infer = 800 frames, i.e. 8
chunks), then ln_post, proj1 + GELU and proj2.  The model definition is
src/qwen_asr/core/transformers_backend/modeling_qwen3_asr.py:451-780.

This module holds the configuration, the host-side input preparation (the same
arithmetic as the reference's), seeded synthetic weights, and AsrEncoderRunner,
which runs the encoder with the library's kernels: conv2d_q8_0 and
linear_q8_0_bias (tensor cores, bias and GELU in the epilogue), layer_norm,
attn_masked (windowed attention as an additive mask), index_rows, add.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from torch2vk_b200 import kernels


@dataclass(frozen=True)
class AsrEncoderConfig:
    num_mel_bins: int = 128
    d_model: int = 896
    layers: int = 18
    heads: int = 14
    ffn: int = 3584
    output_dim: int = 1024
    conv_channels: int = 480
    n_window: int = 50
    n_window_infer: int = 800
    max_source_positions: int = 1500
    eps: float = 1e-5

    @staticmethod
    def qwen3_asr_0_6b() -> "AsrEncoderConfig":
        """Audio tower of Qwen3-ASR-0.6B (the shapes of quantized_qwen3_asr/tensors/audio_encoder.py)."""
        return AsrEncoderConfig()

    @property
    def head_dim(self) -> int:
        return self.d_model // self.heads

    @property
    def freq_after_conv(self) -> int:
        f = self.num_mel_bins
        for _ in range(3):
            f = (f + 1) // 2
        return f

    @property
    def chunk_frames(self) -> int:
        return 2 * self.n_window


def conv_out_len(n: int) -> int:
    """Length after one 3x3 stride-2 padding-1 convolution."""
    return (n + 2 - 3) // 2 + 1


def feat_extract_output_lengths(input_lengths: np.ndarray) -> np.ndarray:
    """Tokens after the convolutions for mel lengths (modeling_qwen3_asr.py:309-317)."""
    input_lengths = np.asarray(input_lengths, dtype=np.int64)
    leave = input_lengths % 100
    feat = (leave - 1) // 2 + 1
    return ((feat - 1) // 2 + 1 - 1) // 2 + 1 + (input_lengths // 100) * 13


def sinusoid_embedding(length: int, channels: int, max_timescale: float = 10000.0) -> np.ndarray:
    """[length, channels] = cat(sin, cos) (SinusoidsPositionEmbedding, modeling_qwen3_asr.py:579-640)."""
    inc = np.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-inc * torch.arange(channels // 2).float())
    t = torch.arange(length)[:, None] * inv[None, :]
    return torch.cat([torch.sin(t), torch.cos(t)], dim=1).numpy().astype(np.float32)


@dataclass
class AsrInputs:
    padded_feature: np.ndarray        # [chunks, 1, n_mel, chunk_frames] fp32
    position_embedding: np.ndarray    # [chunks, t_dim, d_model] fp32
    compact_index: np.ndarray         # [tokens] int64: valid (chunk, t) rows
    cu_seqlens: np.ndarray            # [windows + 1] int32
    attention_mask: np.ndarray        # [1, 1, tokens, tokens] fp32: 0 inside a window, -FLT_MAX outside


def prepare_inputs(mel: np.ndarray, cfg: AsrEncoderConfig) -> AsrInputs:
    """Host preparation of one utterance's log-mel features [n_mel, frames] (pytorch_modules.py:50-110)."""
    mel = np.ascontiguousarray(mel, dtype=np.float32)
    n_mel, feat_len = mel.shape
    cf = cfg.chunk_frames
    chunk_num = int(np.ceil(feat_len / cf))
    chunk_lengths = np.full(chunk_num, cf, dtype=np.int64)
    if feat_len % cf:
        chunk_lengths[-1] = feat_len % cf
    padded = np.zeros((chunk_num, 1, n_mel, cf), dtype=np.float32)
    off = 0
    for i, n in enumerate(chunk_lengths):
        padded[i, 0, :, :n] = mel[:, off:off + n]
        off += int(n)
    t_dim = conv_out_len(conv_out_len(conv_out_len(cf)))
    pos = sinusoid_embedding(cfg.max_source_positions, cfg.d_model)[:t_dim]
    position_embedding = np.ascontiguousarray(np.broadcast_to(pos[None], (chunk_num, t_dim, cfg.d_model)))
    after = feat_extract_output_lengths(chunk_lengths)
    compact = np.array([c * t_dim + t for c, n in enumerate(after) for t in range(int(n))], dtype=np.int64)
    total = int(feat_extract_output_lengths(np.array([feat_len]))[0])
    window = int(after.max()) * (cfg.n_window_infer // cf)
    cu = [0] + [window] * (total // window) + ([total % window] if total % window else [])
    cu_seqlens = np.cumsum(cu, dtype=np.int32)
    n_tok = compact.shape[0]
    mask = np.full((1, 1, n_tok, n_tok), -np.finfo(np.float32).max, dtype=np.float32)
    for i in range(1, len(cu_seqlens)):
        a, b = int(cu_seqlens[i - 1]), int(cu_seqlens[i])
        mask[0, 0, a:b, a:b] = 0.0
    return AsrInputs(padded, position_embedding, compact, cu_seqlens, mask)


# ------------------------------------------------------------------ weights
def param_shapes(cfg: AsrEncoderConfig) -> dict[str, tuple[int, ...]]:
    """Parameter names (those of Qwen3ASRAudioEncoder) and shapes."""
    c, d = cfg.conv_channels, cfg.d_model
    shapes: dict[str, tuple[int, ...]] = {
        "conv2d1.weight": (c, 1, 3, 3), "conv2d1.bias": (c,),
        "conv2d2.weight": (c, c, 3, 3), "conv2d2.bias": (c,),
        "conv2d3.weight": (c, c, 3, 3), "conv2d3.bias": (c,),
        "conv_out.weight": (d, c * cfg.freq_after_conv),
    }
    for i in range(cfg.layers):
        p = f"layers.{i}."
        for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
            shapes[p + f"self_attn.{n}.weight"] = (d, d)
            shapes[p + f"self_attn.{n}.bias"] = (d,)
        for n in ("self_attn_layer_norm", "final_layer_norm"):
            shapes[p + f"{n}.weight"] = (d,)
            shapes[p + f"{n}.bias"] = (d,)
        shapes[p + "fc1.weight"] = (cfg.ffn, d)
        shapes[p + "fc1.bias"] = (cfg.ffn,)
        shapes[p + "fc2.weight"] = (d, cfg.ffn)
        shapes[p + "fc2.bias"] = (d,)
    shapes["ln_post.weight"] = (d,)
    shapes["ln_post.bias"] = (d,)
    shapes["proj1.weight"] = (d, d)
    shapes["proj1.bias"] = (d,)
    shapes["proj2.weight"] = (cfg.output_dim, d)
    shapes["proj2.bias"] = (cfg.output_dim,)
    return shapes


def random_params(cfg: AsrEncoderConfig, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded fp32 parameters (numpy's generator: identical on every machine).

    Linear / conv weights ~ N(0, std), biases ~ N(0, std), LayerNorm weights 1 + N(0, 0.1) and
    biases N(0, 0.02); the convolutions use std * 3 so activations keep unit scale."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in param_shapes(cfg).items():
        if "layer_norm" in name or name.startswith("ln_post"):
            base = 1.0 if name.endswith("weight") else 0.0
            scale = 0.1 if name.endswith("weight") else 0.02
            out[name] = (base + scale * rng.standard_normal(shape)).astype(np.float32)
        else:
            s = std * 3 if name.startswith("conv2d") else std
            out[name] = (s * rng.standard_normal(shape)).astype(np.float32)
    return out


def q8_rows(w: np.ndarray) -> np.ndarray:
    """Weight as the [rows, K] matrix the Q8_0 kernels take: conv [Co, Ci, kh, kw] -> [Co, Ci*kh*kw]
    (k = (ic, fh, fw)), zero-padded along K to whole 32-value blocks."""
    m = w.reshape(w.shape[0], -1)
    k = m.shape[1]
    kp = (k + 31) // 32 * 32
    if kp != k:
        m = np.concatenate([m, np.zeros((m.shape[0], kp - k), dtype=m.dtype)], axis=1)
    return np.ascontiguousarray(m, dtype=np.float32)


def quantized_names(cfg: AsrEncoderConfig) -> list[str]:
    """The Q8_0 tensors (every matrix of the audio tower: quantized_qwen3_asr/quantization.py:8-9)."""
    return [n for n, s in param_shapes(cfg).items() if n.endswith("weight") and len(s) >= 2]


# ------------------------------------------------------------------ runner
class AsrEncoderRunner:
    """The audio encoder on one GPU: Q8_0 weights quantized on the device from fp32 parameters."""

    def __init__(self, cfg: AsrEncoderConfig, params: dict[str, np.ndarray], device: str | torch.device = "cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        qn = set(quantized_names(cfg))
        self.w: dict[str, torch.Tensor] = {}
        # linear weights whose K is not a multiple of 256 (d_model 896 = 28 Q8_0 blocks) get zero blocks up to
        # the next multiple, so the tcgen05 GEMM (256-value TMA windows) takes them; their inputs are padded
        # with zeros to match.  The blocks of the real columns are quantized exactly as before.
        # Convolutions whose Ci * 3 * 3 reaches 256 run as im2col + the same GEMM (conv_kp: their padded K)
        self.kpad: dict[str, int] = {}
        self.conv_kp: dict[str, int] = {}
        for name, arr in params.items():
            if name in qn:
                rows = q8_rows(arr)
                if arr.ndim == 4 and rows.shape[1] >= 256:
                    kp = (rows.shape[1] + 255) // 256 * 256
                    rows = np.concatenate([rows, np.zeros((rows.shape[0], kp - rows.shape[1]), np.float32)], axis=1)
                    self.conv_kp[name] = kp
                elif arr.ndim == 2 and rows.shape[1] % 256:
                    kp = (rows.shape[1] + 255) // 256 * 256
                    rows = np.concatenate([rows, np.zeros((rows.shape[0], kp - rows.shape[1]), np.float32)], axis=1)
                    self.kpad[name] = kp
                t = torch.from_numpy(np.ascontiguousarray(rows)).to(self.device)
                self.w[name] = kernels.quantize(t, "q8_0")
            else:
                self.w[name] = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32)).to(self.device)

    def upload(self, inputs: AsrInputs) -> dict[str, torch.Tensor]:
        dev = self.device
        mask = torch.from_numpy(inputs.attention_mask).to(torch.float16)  # -FLT_MAX becomes -inf in fp16
        return {
            "feature": torch.from_numpy(inputs.padded_feature).to(torch.float16).to(dev),
            "pos": torch.from_numpy(inputs.position_embedding).to(torch.float16).to(dev),
            "index": torch.from_numpy(inputs.compact_index).to(dev),
            "mask": mask.to(dev),
        }

    def forward(self, t: dict[str, torch.Tensor]) -> torch.Tensor:
        """Encoder output rows [tokens, output_dim] fp16 of one uploaded utterance."""
        return self.forward_batch([t])[0]

    def forward_batch(self, clips: list[dict[str, torch.Tensor]]) -> torch.Tensor:
        """Encoder output [B, tokens, output_dim] fp16 of B uploaded utterances of the same length in one
        pass: the convolutions run over all B x chunks, the linears over all B x tokens rows, and the
        windowed attention per utterance (batch B, the same window mask)."""
        cfg, w = self.cfg, self.w
        c, d = cfg.conv_channels, cfg.d_model
        B = len(clips)
        if B == 0:
            raise ValueError("forward_batch needs at least one utterance")
        first = clips[0]
        for t in clips[1:]:
            if t["feature"].shape != first["feature"].shape or t["index"].shape != first["index"].shape:
                raise ValueError("forward_batch: utterances must have the same number of frames")
        cat = (lambda key: first[key]) if B == 1 else (lambda key: torch.cat([t[key] for t in clips], 0))
        x = cat("feature")
        nhwc = False  # x is [bc, C, H, W]; after a GEMM convolution it is [bc, H, W, C]
        for i in (1, 2, 3):
            name = f"conv2d{i}.weight"
            bc = x.shape[0]
            ci, hi, wi = (x.shape[3], x.shape[1], x.shape[2]) if nhwc else (x.shape[1], x.shape[2], x.shape[3])
            if name in self.conv_kp:
                # channels-last input (16-byte gathers of 8 channels), im2col, the tcgen05 GEMM with bias + GELU
                if not nhwc and ci % 8 == 0:
                    xl = torch.empty(bc, hi, wi, ci, dtype=torch.float16, device=x.device)
                    kernels.copy4d(x.permute(0, 2, 3, 1), xl)
                    x, nhwc = xl, True
                sb, s1, s2, s3 = x.stride()
                strides = (sb, s3, s1, s2) if nhwc else (sb, s1, s2, s3)
                cols = kernels.im2col(x, channels=ci, height=hi, width=wi, strides_bchw=strides, batch=bc,
                                      kp=self.conv_kp[name], channels_last=nhwc)
                ho, wo = conv_out_len(hi), conv_out_len(wi)
                x = kernels.linear_q8_0_bias(cols, w[name], w[f"conv2d{i}.bias"], c, gelu=True).view(bc, ho, wo, c)
                nhwc = True
            else:
                if nhwc:
                    xc = torch.empty(bc, ci, hi, wi, dtype=torch.float16, device=x.device)
                    kernels.copy4d(x.permute(0, 3, 1, 2), xc)
                    x, nhwc = xc, False
                # channels-last output when the next convolution is an im2col GEMM (16-byte gathers)
                nxt = f"conv2d{i + 1}.weight"
                cl = nxt in self.conv_kp and c % 8 == 0
                x = kernels.conv2d_q8_0(x, w[name], w[f"conv2d{i}.bias"], c, gelu=True, channels_last_out=cl)
                nhwc = cl
        if nhwc:
            bc, f, td, _ = x.shape
        else:
            bc, _, f, td = x.shape
        chunks = bc // B
        xt = torch.empty(bc, td, c, f, dtype=torch.float16, device=x.device)
        # xt[b, t, c, f]: from [bc, f, td, c] (GEMM) or [bc, c, f, td] (direct convolution)
        kernels.copy4d(x.permute(0, 2, 3, 1) if nhwc else x.permute(0, 3, 1, 2), xt)
        e = kernels.linear_q8_0_bias(xt.view(bc, td, c * f), w["conv_out.weight"], None, d)
        e = kernels.add(e, cat("pos"))
        if B == 1:
            index = first["index"]
        else:
            index = torch.cat([t["index"] + b * chunks * td for b, t in enumerate(clips)], 0)
        h = kernels.index_rows(e.view(bc * td, d), index)
        n = first["index"].shape[0]
        hd = cfg.head_dim
        scale = 1.0 / math.sqrt(hd)
        rows = B * n
        kp = self.kpad.get("layers.0.self_attn.q_proj.weight", d)  # padded width of d-wide linear inputs

        def padded(x: torch.Tensor) -> torch.Tensor:  # [rows, d] -> [rows, kp], zero columns past d
            if kp == d:
                return x
            xp = torch.zeros(rows, kp, dtype=torch.float16, device=x.device)
            kernels.copy4d(x.view(1, 1, rows, d), xp[:, :d].unsqueeze(0).unsqueeze(0))
            return xp

        def lin(x: torch.Tensor, name: str, n_out: int, gelu: bool = False) -> torch.Tensor:
            return kernels.linear_q8_0_bias(x, w[name + ".weight"], w[name + ".bias"], n_out, gelu=gelu)

        def ln(x: torch.Tensor, name: str) -> torch.Tensor:  # LayerNorm into the zero-padded linear input
            return kernels.layer_norm(x, w[name + ".weight"], w[name + ".bias"], cfg.eps, pad_to=kp)

        # the attention writes straight into the (zero-padded) input of out_proj: one buffer for every
        # layer, its padding columns zeroed once
        o = torch.zeros(rows, kp, dtype=torch.float16, device=h.device) if kp != d else \
            torch.empty(rows, d, dtype=torch.float16, device=h.device)

        for i in range(cfg.layers):
            p = f"layers.{i}."
            r = h
            a = ln(h, p + "self_attn_layer_norm")
            q = lin(a, p + "self_attn.q_proj", d)
            k = lin(a, p + "self_attn.k_proj", d)
            v = lin(a, p + "self_attn.v_proj", d)

            def heads(z: torch.Tensor) -> torch.Tensor:  # rows of width z.stride(0) -> [B, H, n, hd] view
                return z.as_strided((B, cfg.heads, n, hd), (n * z.stride(0), hd, z.stride(0), 1))

            kernels.attn_masked(heads(q), heads(k), heads(v), first["mask"], scale=scale, out=heads(o))
            h = kernels.add(r, lin(o, p + "self_attn.out_proj", d))
            r = h
            a = ln(h, p + "final_layer_norm")
            a = lin(a, p + "fc1", cfg.ffn, gelu=True)
            a = lin(a, p + "fc2", d)
            h = kernels.add(r, a)
        h = ln(h, "ln_post")
        h = padded(lin(h, "proj1", d, gelu=True))
        return lin(h, "proj2", cfg.output_dim).view(B, n, -1)

    def flops(self, inputs: AsrInputs) -> float:
        """Multiply-add flops of one forward (convolutions, linears, attention within windows)."""
        cfg = self.cfg
        chunks, _, n_mel, frames = inputs.padded_feature.shape
        c, d = cfg.conv_channels, cfg.d_model
        h1, w1 = conv_out_len(n_mel), conv_out_len(frames)
        h2, w2 = conv_out_len(h1), conv_out_len(w1)
        h3, w3 = conv_out_len(h2), conv_out_len(w2)
        conv = chunks * (h1 * w1 * c * 9 + h2 * w2 * c * c * 9 + h3 * w3 * c * c * 9)
        n = inputs.compact_index.shape[0]
        lin = chunks * w3 * c * h3 * d + cfg.layers * n * (4 * d * d + 2 * d * cfg.ffn) + n * (d * d + d * cfg.output_dim)
        win = np.diff(inputs.cu_seqlens).astype(np.int64)
        attn = cfg.layers * 2 * int((win * win).sum()) * d
        return 2.0 * float(conv + lin + attn)

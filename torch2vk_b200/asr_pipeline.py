"""Qwen3-ASR end to end on one GPU: log-mel clips -> audio encoder -> audio rows
injected into the prompt embedding -> Qwen3 text decoder prefill -> greedy
decode (the reference's driver loop, src/models/optimized_qwen3_asr/run.py:235-440:
audio tower frame, text prefill with audio inject + LM-head select + token
store, then replayed decode steps).

The prompt is [prefix ids] + [one placeholder per audio token] + [suffix ids];
the placeholders' embedding rows are replaced by the encoder's output rows
(the reference's audio_inject program).  The reference builds the prefix and
suffix with the model's chat template; without the tokenizer and checkpoint
in this environment they are caller-supplied ids.  Audio-only prompts use
equal positions in the three multimodal RoPE sections, so the text decoder's
standard RoPE applies (as in the reference's generated code for such prompts).
Batching: B clips of the same length decode together as B sequences.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from torch2vk_b200.asr import AsrEncoderConfig, AsrEncoderRunner, prepare_inputs
from torch2vk_b200.qwen3 import Qwen3Config, Qwen3Runner, Qwen3Weights


@dataclass
class AsrTiming:
    encoder_s: float
    prefill_s: float
    decode_s: float


class AsrPipeline:
    """Encoder and text decoder of a Qwen3-ASR model for `batch` clips of `frames` mel frames each."""

    def __init__(self, enc_cfg: AsrEncoderConfig, enc_params: dict[str, np.ndarray], text_cfg: Qwen3Config,
                 text_weights: Qwen3Weights, *, batch: int, frames: int, prefix: int, suffix: int,
                 max_new_tokens: int = 64, device: str | torch.device = "cuda"):
        if enc_cfg.output_dim != text_cfg.hidden:
            raise ValueError(f"encoder output_dim {enc_cfg.output_dim} != text hidden {text_cfg.hidden}")
        self.device = torch.device(device)
        self.enc_cfg, self.text_cfg = enc_cfg, text_cfg
        self.batch, self.frames = batch, frames
        self.encoder = AsrEncoderRunner(enc_cfg, enc_params, device=self.device)
        probe = prepare_inputs(np.zeros((enc_cfg.num_mel_bins, frames), np.float32), enc_cfg)
        self.audio_tokens = int(probe.compact_index.shape[0])
        self.prefix, self.suffix = prefix, suffix
        self.prompt_len = prefix + self.audio_tokens + suffix
        self.audio_positions = torch.arange(prefix, prefix + self.audio_tokens, dtype=torch.int64, device=self.device)
        self.max_new_tokens = max_new_tokens
        self.runner = Qwen3Runner(text_cfg, text_weights, batch=batch, max_seq=self.prompt_len + max_new_tokens + 8,
                                  max_new_tokens=max_new_tokens + 1)
        self.features = torch.empty(batch, self.audio_tokens, text_cfg.hidden, dtype=torch.float16,
                                    device=self.device)

    def upload(self, mels: list[np.ndarray]) -> list[dict[str, torch.Tensor]]:
        """Host preparation (chunking, padding, position embeddings, window masks) and upload of each clip."""
        if len(mels) != self.batch:
            raise ValueError(f"{len(mels)} clips for a pipeline of batch {self.batch}")
        out = []
        for mel in mels:
            if mel.shape != (self.enc_cfg.num_mel_bins, self.frames):
                raise ValueError(f"mel shape {mel.shape}, expected {(self.enc_cfg.num_mel_bins, self.frames)}")
            out.append(self.encoder.upload(prepare_inputs(np.asarray(mel, np.float32), self.enc_cfg)))
        return out

    def encode(self, clips: list[dict[str, torch.Tensor]]) -> torch.Tensor:
        """All clips through the audio tower in one batched pass (AsrEncoderRunner.forward_batch)."""
        self.features.copy_(self.encoder.forward_batch(clips))
        return self.features

    def prompt(self, prefix_ids: torch.Tensor, suffix_ids: torch.Tensor, placeholder: int) -> torch.Tensor:
        """[batch, prompt_len] ids: prefix, audio placeholders, suffix."""
        b = self.batch
        mid = torch.full((b, self.audio_tokens), placeholder, dtype=torch.int64, device=self.device)
        return torch.cat([prefix_ids.to(self.device).expand(b, -1), mid, suffix_ids.to(self.device).expand(b, -1)],
                         dim=1).contiguous()

    def transcribe(self, clips: list[dict[str, torch.Tensor]], prompt_ids: torch.Tensor) -> torch.Tensor:
        """Greedy token ids [batch, max_new_tokens] (the first from the prefill's LM head)."""
        self.encode(clips)
        self.runner.prefill(prompt_ids, inject=(self.audio_positions, self.features))
        for _ in range(self.max_new_tokens - 1):
            self.runner.step()
        return self.runner.generated[:, :self.max_new_tokens]

    def timed_transcribe(self, clips: list[dict[str, torch.Tensor]], prompt_ids: torch.Tensor) -> AsrTiming:
        """transcribe() with each phase timed by CUDA events on the current stream."""
        stream = torch.cuda.current_stream(self.device)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record(stream)
        self.encode(clips)
        ev[1].record(stream)
        self.runner.prefill(prompt_ids, inject=(self.audio_positions, self.features))
        ev[2].record(stream)
        for _ in range(self.max_new_tokens - 1):
            self.runner.step()
        ev[3].record(stream)
        ev[3].synchronize()
        return AsrTiming(ev[0].elapsed_time(ev[1]) * 1e-3, ev[1].elapsed_time(ev[2]) * 1e-3,
                         ev[2].elapsed_time(ev[3]) * 1e-3)

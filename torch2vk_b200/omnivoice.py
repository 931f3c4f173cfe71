"""OmniVoice LLM forward on one GPU: the per-step forward of OmniVoice's masked
iterative decoding (the reference's generated llm_forward program,
src/models/quantized_omnivoice/dispatch/llm_forward.py, driven by
quantized_omnivoice/run.py:113-129 once per decoding step).

One step: input embedding (text rows, or the sum over the codebooks of audio
rows, both Q8_0; omnivoice_input_embed_q8_0_f32, quantized_omnivoice/
custom_shaders.py:17-181) -> Qwen3 decoder layers with bidirectional attention
under an explicit additive mask (sdpa_masked_f32) -> final RMSNorm -> the
audio heads (Q6_K linear, hidden -> codebooks x audio vocabulary).  The
classifier-free-guidance batch is the reference's: sequence 0 conditional
(style + text + target audio), sequence 1 unconditional (the target audio
alone, padding rows attending only to themselves).

The LLM linears use the Q4_K_M topology (Q6_K v_proj / down_proj in the
more-bits layers, quantized_omnivoice/quantization.py:32-39), the embeddings
Q8_0 (quantization.py:11-27).  CFG scoring, the top-k token update and the
audio codec decoder are not part of this path.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from torch2vk_b200 import _lib, kernels
from torch2vk_b200.qwen3 import LayerWeights, QWeight, Qwen3Config, inv_freq


@dataclass(frozen=True)
class OmniVoiceConfig:
    llm: Qwen3Config
    codebooks: int = 8
    audio_vocab: int = 1025
    audio_mask_id: int = 1024

    @staticmethod
    def omnivoice() -> "OmniVoiceConfig":
        """OmniVoice's LLM is Qwen3-0.6B-shaped (28 layers, hidden 1024, 16 Q / 8 KV heads); the audio heads
        are 8 codebooks x 1025 ids (omnivoice/models/omnivoice.py:169-171; tensors/audio_head.py: [8200, 1024])."""
        return OmniVoiceConfig(llm=Qwen3Config(hidden=1024, layers=28, heads=16, kv_heads=8, head_dim=128,
                                               intermediate=3072, vocab=151676))

    @property
    def head_rows(self) -> int:
        return self.codebooks * self.audio_vocab


@dataclass
class OmniVoiceWeights:
    text_embed: torch.Tensor   # Q8_0 [text vocab, hidden / 32 * 34] bytes
    audio_embed: torch.Tensor  # Q8_0 [codebooks * audio vocab, hidden / 32 * 34] bytes
    layers: list[LayerWeights]
    final_norm: torch.Tensor
    audio_heads: QWeight       # Q6_K [codebooks * audio vocab, hidden]


@dataclass(frozen=True)
class OmniVoiceInputs:
    """Host-side step inputs (quantized_omnivoice/input_prep.py:48-115)."""

    input_ids: np.ndarray      # int64 [2, codebooks, S]
    audio_mask: np.ndarray     # uint32 [2, S]
    attention_mask: np.ndarray  # float16 [2, 1, S, S]: 0 visible, -inf masked
    target_len: int
    cond_audio_start: int


def prepare_inputs(style_ids: np.ndarray, text_ids: np.ndarray, target_len: int,
                   cfg: OmniVoiceConfig) -> OmniVoiceInputs:
    """The CFG batch of one utterance: sequence 0 = style + text + target_len masked audio positions (every
    row attends to every row), sequence 1 = the target audio positions alone at the front, its padding rows
    attending only to themselves.  style_ids / text_ids are the tokenizer's ids (1-D), repeated over the
    codebooks as the reference does."""
    C = cfg.codebooks
    style = np.broadcast_to(np.asarray(style_ids, np.int64)[None, :], (C, len(style_ids)))
    text = np.broadcast_to(np.asarray(text_ids, np.int64)[None, :], (C, len(text_ids)))
    target = np.full((C, target_len), cfg.audio_mask_id, np.int64)
    cond = np.concatenate([style, text, target], axis=1)
    S = cond.shape[1]
    start = S - target_len
    ids = np.full((2, C, S), cfg.audio_mask_id, np.int64)
    amask = np.zeros((2, S), np.uint32)
    visible = np.zeros((2, 1, S, S), bool)
    ids[0] = cond
    amask[0, start:] = 1
    visible[0, :, :, :] = True
    ids[1, :, :target_len] = cond[:, start:]
    amask[1, :target_len] = 1
    visible[1, :, :target_len, :target_len] = True
    pad = np.arange(target_len, S)
    visible[1, :, pad, pad] = True
    mask = np.where(visible, np.float16(0), np.float16(-np.inf)).astype(np.float16)
    return OmniVoiceInputs(ids, amask, mask, target_len, start)


@dataclass
class OmniVoiceLLM:
    """Static-shape LLM forward for `batch` sequences of `seq` positions (the CFG pair: batch 2)."""

    cfg: OmniVoiceConfig
    weights: OmniVoiceWeights
    batch: int
    seq: int
    _graph: torch.cuda.CUDAGraph | None = field(default=None, init=False)

    def __post_init__(self) -> None:
        c, dev = self.cfg.llm, self.weights.final_norm.device
        self.device = dev
        B, S = self.batch, self.seq
        f16 = dict(dtype=torch.float16, device=dev)
        t = B * S
        self.ids = torch.zeros(B, self.cfg.codebooks, S, dtype=torch.int64, device=dev)
        self.audio_mask = torch.zeros(B, S, dtype=torch.int32, device=dev)
        self.mask = torch.zeros(B, 1, S, S, **f16)
        self.h = torch.empty(t, c.hidden, **f16)
        self.q = torch.empty(t, c.heads * c.head_dim, **f16)
        self.k = torch.empty(t, c.kv_heads * c.head_dim, **f16)
        self.v = torch.empty(t, c.kv_heads * c.head_dim, **f16)
        self.qr = torch.empty(t, c.heads * c.head_dim, **f16)
        self.attn = torch.empty(t, c.heads * c.head_dim, **f16)
        self.act = torch.empty(t, c.intermediate, **f16)
        self.kr = torch.empty(B, S, c.kv_heads, c.head_dim, **f16)
        self.vr = torch.empty(B, S, c.kv_heads, c.head_dim, **f16)
        self.normed = torch.empty(t, c.hidden, **f16)
        self.logits = torch.empty(B, S, self.cfg.head_rows, **f16)
        self.positions = torch.zeros(B, dtype=torch.int32, device=dev)
        self.inv_freq = inv_freq(c).to(dev)

    def upload(self, inputs: OmniVoiceInputs) -> None:
        """Copies one step's host inputs into the static device buffers."""
        if inputs.input_ids.shape != tuple(self.ids.shape):
            raise ValueError(f"input_ids {inputs.input_ids.shape} != {tuple(self.ids.shape)}")
        self.ids.copy_(torch.from_numpy(inputs.input_ids))
        self.audio_mask.copy_(torch.from_numpy(inputs.audio_mask.astype(np.int32)))
        self.mask.copy_(torch.from_numpy(inputs.attention_mask))

    def _embed(self) -> None:
        c = self.cfg
        _lib.lib().call("t2c_omnivoice_input_embed", _lib.ptr(self.weights.text_embed),
                        _lib.ptr(self.weights.audio_embed), _lib.ptr(self.ids), _lib.ptr(self.audio_mask),
                        _lib.ptr(self.h), self.batch, c.codebooks, self.seq, c.llm.hidden, c.llm.vocab,
                        c.audio_vocab, _lib.stream_ptr())

    def _layer(self, lw: LayerWeights) -> None:
        c = self.cfg.llm
        B, S = self.batch, self.seq
        kernels.linear_multi(self.h, [(lw.q.data, lw.q.kind), (lw.k.data, lw.k.kind), (lw.v.data, lw.v.kind)],
                             c.hidden, norm_weight=lw.input_norm, eps=c.eps, outs=[self.q, self.k, self.v])
        kernels.qk_norm_rope_cache(self.q, self.k, self.v, lw.q_norm, lw.k_norm, self.kr, self.vr, self.positions,
                                   self.inv_freq, batch=B, tokens=S, n_heads=c.heads, n_kv=c.kv_heads,
                                   head_dim=c.head_dim, eps=c.eps, q_out=self.qr)
        kernels.attn_masked_gqa(self.qr, self.kr, self.vr, self.mask, batch=B, tokens=S, n_heads=c.heads,
                                n_kv=c.kv_heads, head_dim=c.head_dim, out=self.attn)
        kernels.linear(self.attn, lw.o.data, lw.o.kind, c.heads * c.head_dim, residual=self.h, out=self.h)
        kernels.linear_swiglu(self.h, lw.gate.data, lw.up.data, lw.gate.kind, c.hidden, norm_weight=lw.post_norm,
                              eps=c.eps, out=self.act)
        kernels.linear(self.act, lw.down.data, lw.down.kind, c.intermediate, residual=self.h, out=self.h)

    def forward_device(self, *, layer_outputs: list[torch.Tensor] | None = None) -> torch.Tensor:
        """Embedding, layers, final norm and audio heads over the uploaded inputs: logits [B, S, C * V]."""
        c = self.cfg.llm
        self._embed()
        for lw in self.weights.layers:
            self._layer(lw)
            if layer_outputs is not None:
                layer_outputs.append(self.h.clone())
        kernels.rms_norm(self.h, self.weights.final_norm, c.eps, out=self.normed)
        hd = self.weights.audio_heads
        kernels.linear(self.normed, hd.data, hd.kind, c.hidden, out=self.logits.view(-1, self.cfg.head_rows))
        return self.logits

    def capture(self) -> None:
        """Captures forward_device in a CUDA graph (the reference replays its generation step)."""
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.forward_device()
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self.forward_device()
        self._graph = graph

    def forward(self, inputs: OmniVoiceInputs | None = None) -> torch.Tensor:
        """Graph-replayed step (inputs uploaded first when given)."""
        if inputs is not None:
            self.upload(inputs)
        if self._graph is None:
            self.capture()
        self._graph.replay()
        return self.logits


def random_weights(cfg: OmniVoiceConfig, *, seed: int = 0, device: str = "cuda") -> OmniVoiceWeights:
    """Seeded N(0, 0.02) weights quantized on the GPU with the OmniVoice topology (for timing)."""
    from torch2vk_b200.qwen3 import q4_k_m_more_bits_layers

    c = cfg.llm
    g = torch.Generator(device=device).manual_seed(seed)

    def rnd(*shape: int) -> torch.Tensor:
        return torch.randn(*shape, generator=g, device=device) * 0.02

    def quant(x: torch.Tensor, kind: str) -> QWeight:
        return QWeight(kernels.quantize(x, kind), kind)

    q6 = set(q4_k_m_more_bits_layers(c.layers))
    layers = []
    for i in range(c.layers):
        vk = "q6_k" if i in q6 else "q4_k"
        layers.append(LayerWeights(
            input_norm=torch.ones(c.hidden, device=device), q=quant(rnd(c.heads * c.head_dim, c.hidden), "q4_k"),
            k=quant(rnd(c.kv_heads * c.head_dim, c.hidden), "q4_k"),
            v=quant(rnd(c.kv_heads * c.head_dim, c.hidden), vk), q_norm=torch.ones(c.head_dim, device=device),
            k_norm=torch.ones(c.head_dim, device=device), o=quant(rnd(c.hidden, c.heads * c.head_dim), "q4_k"),
            post_norm=torch.ones(c.hidden, device=device), gate=quant(rnd(c.intermediate, c.hidden), "q4_k"),
            up=quant(rnd(c.intermediate, c.hidden), "q4_k"), down=quant(rnd(c.hidden, c.intermediate), vk)))
    return OmniVoiceWeights(text_embed=kernels.quantize(rnd(c.vocab, c.hidden), "q8_0"),
                            audio_embed=kernels.quantize(rnd(cfg.head_rows, c.hidden), "q8_0"), layers=layers,
                            final_norm=torch.ones(c.hidden, device=device),
                            audio_heads=quant(rnd(cfg.head_rows, c.hidden), "q6_k"))

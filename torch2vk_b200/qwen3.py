"""Qwen3 decoder on the sm_100a kernels: prefill, decode step, greedy generate.

This is the B200 counterpart of the reference's Qwen3 runner
(src/models/quantized_qwen3/run.py:96-415 and the generated
dispatch/decode_layer.py / dispatch/text_layer.py): the same per-layer math
(RMSNorm -> q/k/v -> q/k-norm + RoPE -> attention over the KV cache -> o_proj
+ residual -> RMSNorm -> SwiGLU MLP + residual; final norm -> LM head greedy
select -> token store), fused into six kernels per layer:

  1. fused QKV quantized matvec with the input RMSNorm as prologue
  2. q/k RMSNorm + RoPE + KV-cache write
  3. attention (split-K decode, causal prefill)
  4. o_proj + residual
  5. gate/up + SwiGLU with the post-attention RMSNorm as prologue
  6. down_proj + residual

Weights stay in the GGUF packed layout the reference quantizer produces
(Q4_K / Q6_K / Q8_0 rows, F16 embeddings, F32 norms).  One decode step is
captured in a CUDA graph (the equivalent of the reference's replay plan,
src/torch2vk/runtime/replay.py:163-314); positions and the token index live in
device memory and advance inside the graph.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from torch2vk_b200 import kernels
from torch2vk_b200.paged_kv import PagedKVCache

Q6_NAMES = ("v_proj", "down_proj")


@dataclass(frozen=True)
class Qwen3Config:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    eps: float = 1e-6
    theta: float = 1e6

    @staticmethod
    def qwen3_0_6b() -> "Qwen3Config":
        return Qwen3Config(hidden=1024, layers=28, heads=16, kv_heads=8, head_dim=128, intermediate=3072, vocab=151936)

    @staticmethod
    def qwen3_8b() -> "Qwen3Config":
        return Qwen3Config(hidden=4096, layers=36, heads=32, kv_heads=8, head_dim=128, intermediate=12288, vocab=151936)


def q4_k_m_more_bits_layers(num_layers: int) -> tuple[int, ...]:
    """Layers whose v_proj/down_proj use Q6_K under Q4_K_M (quantize/gguf.py:150-161)."""
    first = num_layers // 8
    last = (7 * num_layers) // 8
    return tuple(i for i in range(num_layers) if i < first or i >= last or (i - first) % 3 == 2)


@dataclass
class QWeight:
    """A packed GGUF weight on the device: data + block type (q4_k / q6_k / q8_0)."""

    data: torch.Tensor
    kind: str


@dataclass
class LayerWeights:
    input_norm: torch.Tensor
    q: QWeight
    k: QWeight
    v: QWeight
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o: QWeight
    post_norm: torch.Tensor
    gate: QWeight
    up: QWeight
    down: QWeight


@dataclass
class Qwen3Weights:
    embed: torch.Tensor          # F16 [vocab, hidden] (or Q4_K packed)
    embed_kind: str
    layers: list[LayerWeights]
    final_norm: torch.Tensor
    lm_head: QWeight


def inv_freq(cfg: Qwen3Config) -> torch.Tensor:
    """RoPE inverse frequencies exactly as the HF Qwen3 rotary embedding computes them (fp32, CPU)."""
    exponent = torch.arange(0, cfg.head_dim, 2, dtype=torch.int64).to(dtype=torch.float32) / cfg.head_dim
    return 1.0 / (cfg.theta ** exponent)


@dataclass
class _Buffers:
    h: torch.Tensor
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    qr: torch.Tensor
    attn: torch.Tensor
    act: torch.Tensor
    ps: torch.Tensor
    pt: torch.Tensor


@dataclass
class Qwen3Runner:
    """Owns the KV cache, activations and the captured decode graph for `batch` sequences."""

    cfg: Qwen3Config
    weights: Qwen3Weights
    batch: int
    max_seq: int
    max_new_tokens: int = 256
    eos_ids: tuple[int, ...] = ()
    decode_splits: int = 0
    fused_attention: bool = True
    page_size: int = 0
    kv_pages: int = 0
    k_cache: list[torch.Tensor] = field(init=False)
    v_cache: list[torch.Tensor] = field(init=False)

    def __post_init__(self) -> None:
        """page_size > 0 keeps the KV cache in a paged pool (PagedKVCache) of kv_pages pages (default: enough
        for every sequence at max_seq) instead of one contiguous [batch, max_seq] cache per layer."""
        cfg, dev = self.cfg, self.weights.final_norm.device
        self.device = dev
        self.paged: PagedKVCache | None = None
        if self.page_size > 0:
            per_seq = -(-self.max_seq // self.page_size)
            self.paged = PagedKVCache(layers=cfg.layers, num_pages=self.kv_pages or self.batch * per_seq,
                                      page_size=self.page_size, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                                      max_seqs=self.batch, max_pages_per_seq=per_seq, device=dev)
            self.k_cache, self.v_cache = self.paged.k, self.paged.v
            # the decode step's new K/V rows, written here by the RoPE kernel (position stride 0) and then
            # copied into their pages
            stage = (self.batch, cfg.kv_heads * cfg.head_dim)
            self.k_stage = torch.zeros(stage, dtype=torch.float16, device=dev)
            self.v_stage = torch.zeros(stage, dtype=torch.float16, device=dev)
        else:
            shape = (self.batch, self.max_seq, cfg.kv_heads, cfg.head_dim)
            self.k_cache = [torch.zeros(shape, dtype=torch.float16, device=dev) for _ in range(cfg.layers)]
            self.v_cache = [torch.zeros(shape, dtype=torch.float16, device=dev) for _ in range(cfg.layers)]
        self.inv_freq = inv_freq(cfg).to(dev)
        self.positions = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self.token_index = torch.zeros(1, dtype=torch.int32, device=dev)
        self.next_token = torch.zeros(self.batch, dtype=torch.int64, device=dev)
        self.done = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self.generated = torch.zeros(self.batch, self.max_new_tokens, dtype=torch.int64, device=dev)
        self.generated_length = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self.stopped = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self.eos = torch.tensor(list(self.eos_ids) or [-1], dtype=torch.int64, device=dev)
        if self.decode_splits <= 0:
            if self.paged is not None:
                want = max(1, 592 // max(1, self.batch * cfg.kv_heads))
                self.decode_splits = max(1, min(32, want, self.max_seq // 64))
            elif self.fused_attention and self.max_seq <= 16384:
                # one cluster of up to 8 CTAs per (sequence, KV head), about two CTAs per SM
                want = max(1, 296 // max(1, self.batch * cfg.kv_heads))
                self.decode_splits = max(1, min(8, want, self.max_seq // 64))
            elif self.fused_attention:
                # long caches: more splits, combined through a global workspace
                want = max(1, 592 // max(1, self.batch * cfg.kv_heads))
                self.decode_splits = max(1, min(32, want, self.max_seq // 64))
            else:
                self.decode_splits = max(1, min(64, self.max_seq // 128))
        ws = kernels.attn_decode_workspace_floats(self.batch, cfg.heads, cfg.head_dim, self.decode_splits)
        self.attn_workspace = torch.empty(max(ws, 1), dtype=torch.float32, device=dev)
        self.fused_workspace = kernels.attn_decode_fused_workspace(self.batch, cfg.heads, cfg.kv_heads, cfg.head_dim,
                                                                   self.decode_splits, dev)
        self.decode = self._alloc(self.batch)
        self._prefill_buffers: tuple[int, _Buffers] | None = None
        self._graph: torch.cuda.CUDAGraph | None = None

    # ------------------------------------------------------------ buffers
    def _alloc(self, tokens: int) -> _Buffers:
        cfg, dev = self.cfg, self.device
        f16 = dict(dtype=torch.float16, device=dev)
        groups = (cfg.vocab + 3) // 4
        rows = self.batch
        return _Buffers(
            h=torch.empty(tokens, cfg.hidden, **f16),
            q=torch.empty(tokens, cfg.heads * cfg.head_dim, **f16),
            k=torch.empty(tokens, cfg.kv_heads * cfg.head_dim, **f16),
            v=torch.empty(tokens, cfg.kv_heads * cfg.head_dim, **f16),
            qr=torch.empty(tokens, cfg.heads * cfg.head_dim, **f16),
            attn=torch.empty(tokens, cfg.heads * cfg.head_dim, **f16),
            act=torch.empty(tokens, cfg.intermediate, **f16),
            ps=torch.empty(rows, groups, dtype=torch.float32, device=dev),
            pt=torch.empty(rows, groups, dtype=torch.int32, device=dev),
        )

    # -------------------------------------------------------------- layers
    def _layer(self, i: int, b: _Buffers, tokens_per_seq: int, decode: bool) -> None:
        cfg, lw = self.cfg, self.weights.layers[i]
        h = b.h
        kernels.linear_multi(h, [(lw.q.data, lw.q.kind), (lw.k.data, lw.k.kind), (lw.v.data, lw.v.kind)], cfg.hidden,
                             norm_weight=lw.input_norm, eps=cfg.eps, outs=[b.q, b.k, b.v])
        self._attention(i, b, tokens_per_seq, decode)
        kernels.linear(b.attn, lw.o.data, lw.o.kind, cfg.heads * cfg.head_dim, residual=h, out=h)
        kernels.linear_swiglu(h, lw.gate.data, lw.up.data, lw.gate.kind, cfg.hidden, norm_weight=lw.post_norm,
                              eps=cfg.eps, out=b.act)
        kernels.linear(b.act, lw.down.data, lw.down.kind, cfg.intermediate, residual=h, out=h)

    def _attention(self, i: int, b: _Buffers, tokens_per_seq: int, decode: bool) -> None:
        """q/k norm + RoPE, KV-cache write and attention of layer i: b.q/b.k/b.v -> b.attn."""
        cfg, lw = self.cfg, self.weights.layers[i]
        if self.paged is not None:
            self._attention_paged(i, b, tokens_per_seq, decode)
            return
        if decode and self.fused_attention:
            kernels.attn_decode_fused(b.q, b.k, b.v, lw.q_norm, lw.k_norm, self.inv_freq, self.k_cache[i],
                                      self.v_cache[i], self.positions, batch=self.batch, n_heads=cfg.heads,
                                      n_kv=cfg.kv_heads, head_dim=cfg.head_dim, splits=self.decode_splits,
                                      workspace=self.fused_workspace, eps=cfg.eps, out=b.attn)
            return
        kernels.qk_norm_rope_cache(b.q, b.k, b.v, lw.q_norm, lw.k_norm, self.k_cache[i], self.v_cache[i],
                                   self.positions, self.inv_freq, batch=self.batch, tokens=tokens_per_seq,
                                   n_heads=cfg.heads, n_kv=cfg.kv_heads, head_dim=cfg.head_dim, eps=cfg.eps,
                                   q_out=b.qr)
        if decode:
            kernels.attn_decode(b.qr, self.k_cache[i], self.v_cache[i], self.positions, batch=self.batch,
                                n_heads=cfg.heads, n_kv=cfg.kv_heads, head_dim=cfg.head_dim, max_len=self.max_seq,
                                splits=self.decode_splits, workspace=self.attn_workspace, out=b.attn)
        else:
            kernels.attn_prefill(b.qr, self.k_cache[i], self.v_cache[i], self.positions, batch=self.batch,
                                 tokens=tokens_per_seq, n_heads=cfg.heads, n_kv=cfg.kv_heads, head_dim=cfg.head_dim,
                                 out=b.attn)

    def _attention_paged(self, i: int, b: _Buffers, tokens_per_seq: int, decode: bool) -> None:
        """_attention over the paged pool.  Decode: RoPE into the staging rows, paged write, paged split-K
        attention.  Prefill (positions start at 0): RoPE into a contiguous prompt cache, causal attention
        over it, then the prompt's rows are copied into their pages."""
        cfg, lw, pool = self.cfg, self.weights.layers[i], self.paged
        nk, d, bt = cfg.kv_heads, cfg.head_dim, pool.block_table
        if decode:
            ks = self.k_stage.as_strided((self.batch, self.max_seq, nk, d), (nk * d, 0, d, 1))
            vs = self.v_stage.as_strided((self.batch, self.max_seq, nk, d), (nk * d, 0, d, 1))
        else:
            ks = torch.empty(self.batch, tokens_per_seq, nk, d, dtype=torch.float16, device=self.device)
            vs = torch.empty_like(ks)
        kernels.qk_norm_rope_cache(b.q, b.k, b.v, lw.q_norm, lw.k_norm, ks, vs, self.positions, self.inv_freq,
                                   batch=self.batch, tokens=tokens_per_seq, n_heads=cfg.heads, n_kv=nk, head_dim=d,
                                   eps=cfg.eps, q_out=b.qr)
        src_k = self.k_stage if decode else ks.view(self.batch, tokens_per_seq, nk * d)
        src_v = self.v_stage if decode else vs.view(self.batch, tokens_per_seq, nk * d)
        for pages, src in ((pool.k[i], src_k), (pool.v[i], src_v)):
            kernels.kv_cache_write_paged(pages, src, self.positions, bt, batch=self.batch, tokens=tokens_per_seq,
                                         n_kv=nk, head_dim=d)
        if decode:
            kernels.attn_decode_paged(b.qr, pool.k[i], pool.v[i], self.positions, bt, batch=self.batch,
                                      n_heads=cfg.heads, n_kv=nk, head_dim=d, splits=self.decode_splits,
                                      workspace=self.attn_workspace, out=b.attn)
        else:
            kernels.attn_prefill(b.qr, ks, vs, self.positions, batch=self.batch, tokens=tokens_per_seq,
                                 n_heads=cfg.heads, n_kv=nk, head_dim=d, out=b.attn)

    def _reserve_pages(self, positions: int) -> None:
        """Every sequence gets pages for `positions` positions, handed out round-robin (sequence b's pages
        are then not adjacent in the pool); pages held from an earlier prompt are returned first."""
        pool = self.paged
        for s in range(self.batch):
            pool.release(s)
        for end in range(pool.page_size, positions + pool.page_size, pool.page_size):
            for s in range(self.batch):
                pool.reserve(s, min(end, positions))

    def _embed(self, ids: torch.Tensor, out: torch.Tensor) -> None:
        cfg = self.cfg
        kernels.embedding(self.weights.embed, self.weights.embed_kind, ids, cfg.hidden, cfg.vocab, out=out)

    def _head(self, x_last: torch.Tensor, b: _Buffers) -> None:
        cfg, w = self.cfg, self.weights
        kernels.lm_head_argmax(x_last, w.lm_head.data, w.lm_head.kind, cfg.hidden, norm_weight=w.final_norm,
                               eps=cfg.eps, partial_scores=b.ps, partial_tokens=b.pt)
        kernels.token_select(b.ps, b.pt, self.eos, next_token=self.next_token, done=self.done)
        kernels.token_store(self.next_token, self.done, self.generated, self.generated_length, self.stopped,
                            token_index_dev=self.token_index, stop_on_eos=bool(self.eos_ids))

    # ------------------------------------------------------------- forward
    def prefill(self, ids: torch.Tensor, *, layer_outputs: list[torch.Tensor] | None = None,
                inject: tuple[torch.Tensor, torch.Tensor] | None = None) -> None:
        """Runs the prompt ids [batch, T] through all layers and selects the first new token.

        inject = (positions int64 [S], rows fp16 [batch, S, hidden]): after the token embedding, the
        rows at those prompt positions are replaced (Qwen3-ASR's audio features at the audio placeholder
        positions: the reference's audio_inject program, optimized_qwen3_asr/dispatch)."""
        cfg = self.cfg
        if ids.shape[0] != self.batch:
            raise ValueError(f"prefill ids batch {ids.shape[0]} != runner batch {self.batch}")
        tokens = ids.shape[1]
        if tokens > self.max_seq:
            raise ValueError(f"prompt of {tokens} tokens exceeds max_seq {self.max_seq}")
        if self.paged is not None:
            self._reserve_pages(min(self.max_seq, tokens + self.max_new_tokens))
        self.positions.zero_()
        self.token_index.zero_()
        self.generated_length.zero_()
        self.stopped.zero_()
        # prompt-sized activations are kept for the next prefill of the same length (no allocator traffic
        # on repeated prompts)
        if self._prefill_buffers is None or self._prefill_buffers[0] != tokens:
            self._prefill_buffers = None
            self._prefill_buffers = (tokens, self._alloc(self.batch * tokens))
        b = self._prefill_buffers[1]
        self._embed(ids.reshape(-1).contiguous(), b.h)
        if inject is not None:
            kernels.index_copy_rows(b.h.view(self.batch, tokens, cfg.hidden), inject[0], inject[1])
        for i in range(cfg.layers):
            self._layer(i, b, tokens, decode=False)
            if layer_outputs is not None:
                layer_outputs.append(b.h.clone())
        last = b.h.view(self.batch, tokens, cfg.hidden)[:, -1, :].contiguous()
        self._head(last, b)
        self.positions.fill_(tokens)
        self.token_index.fill_(1)

    def decode_step(self, *, layer_outputs: list[torch.Tensor] | None = None) -> None:
        """One greedy token for every sequence: embeds next_token, appends the new one."""
        cfg, b = self.cfg, self.decode
        self._embed(self.next_token, b.h)
        for i in range(cfg.layers):
            self._layer(i, b, 1, decode=True)
            if layer_outputs is not None:
                layer_outputs.append(b.h.clone())
        self._head(b.h, b)
        kernels.advance_positions(self.positions, self.token_index)

    def _step_state(self) -> list[torch.Tensor]:
        return [self.positions, self.token_index, self.next_token, self.done, self.generated, self.generated_length,
                self.stopped]

    def capture(self) -> None:
        """Captures decode_step in a CUDA graph (replayed by step()).

        The warm-up run and the capture both execute decode_step once, so every
        piece of step state is saved before and restored after (the KV-cache row
        they write is rewritten by the first replay).
        """
        saved = [t.clone() for t in self._step_state()]
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.decode_step()  # warm up every launch path outside capture
        torch.cuda.current_stream(self.device).wait_stream(side)
        for t, v in zip(self._step_state(), saved):
            t.copy_(v)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self.decode_step()
        self._graph = graph
        for t, v in zip(self._step_state(), saved):
            t.copy_(v)

    def step(self) -> None:
        if self._graph is None:
            self.capture()
        self._graph.replay()

    def generate(self, prompt: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
        """Prefill + (max_new_tokens - 1) graph-replayed decode steps; returns [batch, max_new_tokens]."""
        if max_new_tokens > self.max_new_tokens:
            raise ValueError(f"max_new_tokens {max_new_tokens} > capacity {self.max_new_tokens}")
        if prompt.shape[1] + max_new_tokens > self.max_seq:
            raise ValueError("prompt + new tokens exceed max_seq")
        self.prefill(prompt)
        for _ in range(max_new_tokens - 1):
            self.step()
        return self.generated[:, :max_new_tokens]


# ------------------------------------------------------------------ weights
def _quant(x: torch.Tensor, kind: str) -> QWeight:
    return QWeight(kernels.quantize(x.float().contiguous(), kind), kind)


def random_weights(cfg: Qwen3Config, *, seed: int = 0, device: str = "cuda", lm_head_kind: str = "q6_k",
                   topology: str = "q4_k", std: float = 0.02) -> Qwen3Weights:
    """Seeded N(0, std) weights generated and quantized on the GPU (norms = 1).

    topology "q4_k": every linear Q4_K; "q4_k_m": v_proj/down_proj of the
    Q4_K_M more-bits layers Q6_K (quantize/gguf.py:150-161).  Embeddings F16.
    """
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)

    def rnd(*shape: int) -> torch.Tensor:
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std

    q6_layers = set(q4_k_m_more_bits_layers(cfg.layers)) if topology == "q4_k_m" else set()
    ones = lambda n: torch.ones(n, dtype=torch.float32, device=device)  # noqa: E731
    embed_f32 = rnd(cfg.vocab, cfg.hidden)
    layers = []
    for i in range(cfg.layers):
        kv_kind = "q6_k" if i in q6_layers else "q4_k"
        layers.append(LayerWeights(
            input_norm=ones(cfg.hidden),
            q=_quant(rnd(cfg.heads * cfg.head_dim, cfg.hidden), "q4_k"),
            k=_quant(rnd(cfg.kv_heads * cfg.head_dim, cfg.hidden), "q4_k"),
            v=_quant(rnd(cfg.kv_heads * cfg.head_dim, cfg.hidden), kv_kind),
            q_norm=ones(cfg.head_dim),
            k_norm=ones(cfg.head_dim),
            o=_quant(rnd(cfg.hidden, cfg.heads * cfg.head_dim), "q4_k"),
            post_norm=ones(cfg.hidden),
            gate=_quant(rnd(cfg.intermediate, cfg.hidden), "q4_k"),
            up=_quant(rnd(cfg.intermediate, cfg.hidden), "q4_k"),
            down=_quant(rnd(cfg.hidden, cfg.intermediate), kv_kind),
        ))
    lm_head = _quant(embed_f32, lm_head_kind)
    return Qwen3Weights(embed=embed_f32.half(), embed_kind="f16", layers=layers, final_norm=ones(cfg.hidden),
                        lm_head=lm_head)


def weight_bytes(w: Qwen3Weights) -> dict[str, int]:
    """Bytes one decode step streams for the weights (linears, lm head)."""
    lin = 0
    for lw in w.layers:
        for q in (lw.q, lw.k, lw.v, lw.o, lw.gate, lw.up, lw.down):
            lin += q.data.numel() * q.data.element_size()
    head = w.lm_head.data.numel() * w.lm_head.data.element_size()
    return {"linears": lin, "lm_head": head}

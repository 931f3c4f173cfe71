"""Tensor parallelism for the Qwen3 decoder: one process per GPU, NCCL over NVLink.

Megatron-style split of one layer over `tp` ranks (the plan of the hot-path
survey for Qwen3-8B):
  * q / k / v: column-split by heads (NH/tp query heads, NK/tp KV heads per
    rank; the GQA groups stay whole), KV cache sharded by KV head;
  * o_proj, down_proj: row-split along K (the packed Q4_K rows are cut at
    super-block boundaries: K/tp must be a multiple of 256); rank 0 adds the
    residual, then one all-reduce of the fp16 hidden state per sub-block;
  * gate / up: column-split (I/tp rows per rank), SwiGLU local;
  * LM head: vocab-split (V/tp rows, multiple of 4); every rank computes its
    argmax partials, the partials (with global token ids) are all-gathered
    and every rank runs the same final select, so the sampled token is
    identical everywhere;
  * embedding, norms: replicated.
Two all-reduces per layer ([tokens, hidden] fp16) and one all-gather per step.
With fused_reduce the two reductions at one token run inside the o_proj /
down_proj matvecs (t2c_linear_allreduce: fp32 partials pushed over NVLink peer
memory, one flag round trip per CTA, summed in rank order, residual added);
otherwise decode-sized all-reduces run as one kernel over NVLink peer memory
(torch2vk_b200.comm, CUDA IPC buffers, bounded flag waits); larger ones
(prefill) and the all-gather use NCCL.  Every collective is issued on the
runner's stream, so a decode step with its collectives is captured in one
CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from torch2vk_b200 import kernels
from torch2vk_b200.qwen3 import LayerWeights, QWeight, Qwen3Config, Qwen3Runner, Qwen3Weights

BLOCK_BYTES = {"q4_k": (256, 144), "q6_k": (256, 210), "q8_0": (32, 34)}


def shard_rows(w: QWeight, rank: int, tp: int) -> QWeight:
    """Rows [rank * N/tp, (rank+1) * N/tp) of a packed weight (column-parallel split)."""
    n = w.data.shape[0]
    if n % tp:
        raise ValueError(f"{n} rows do not split over {tp} ranks")
    rows = n // tp
    return QWeight(w.data[rank * rows:(rank + 1) * rows].contiguous(), w.kind)


def shard_k(w: QWeight, k: int, rank: int, tp: int) -> QWeight:
    """Columns [rank * K/tp, (rank+1) * K/tp) of every row of a packed weight (row-parallel split)."""
    values, nbytes = BLOCK_BYTES[w.kind]
    if k % (tp * values):
        raise ValueError(f"K={k} does not split over {tp} ranks at {values}-value blocks")
    raw = w.data.view(torch.uint8).reshape(w.data.shape[0], -1)
    part = raw.shape[1] // tp
    if part * tp != raw.shape[1]:
        raise ValueError("packed row bytes do not split evenly")
    piece = raw[:, rank * part:(rank + 1) * part].contiguous()
    return QWeight(piece.view(w.data.dtype), w.kind)


def local_config(cfg: Qwen3Config, tp: int) -> Qwen3Config:
    if cfg.heads % tp or cfg.kv_heads % tp or cfg.intermediate % tp or cfg.vocab % (4 * tp):
        raise ValueError(f"Qwen3 config does not split over {tp} ranks")
    return replace(cfg, heads=cfg.heads // tp, kv_heads=cfg.kv_heads // tp, intermediate=cfg.intermediate // tp,
                   vocab=cfg.vocab // tp)


def shard_weights(w: Qwen3Weights, cfg: Qwen3Config, rank: int, tp: int) -> Qwen3Weights:
    """This rank's part of full Qwen3 weights (all tensors already on this rank's device)."""
    layers = []
    for lw in w.layers:
        layers.append(LayerWeights(
            input_norm=lw.input_norm, q=shard_rows(lw.q, rank, tp), k=shard_rows(lw.k, rank, tp),
            v=shard_rows(lw.v, rank, tp), q_norm=lw.q_norm, k_norm=lw.k_norm,
            o=shard_k(lw.o, cfg.heads * cfg.head_dim, rank, tp), post_norm=lw.post_norm,
            gate=shard_rows(lw.gate, rank, tp), up=shard_rows(lw.up, rank, tp),
            down=shard_k(lw.down, cfg.intermediate, rank, tp)))
    return Qwen3Weights(embed=w.embed, embed_kind=w.embed_kind, layers=layers, final_norm=w.final_norm,
                        lm_head=shard_rows(w.lm_head, rank, tp))


@dataclass
class TPQwen3Runner(Qwen3Runner):
    """Qwen3Runner over `tp` ranks: weights / KV heads local, hidden state replicated."""

    full_cfg: Qwen3Config | None = None
    rank: int = 0
    tp: int = 1
    group: object | None = None
    peer_allreduce: bool = True  # decode-sized reductions over NVLink peer memory instead of NCCL
    # 1-token o_proj / down_proj with the reduction inside the matvec's epilogue (t2c_linear_allreduce).
    # Off by default: measured at TP = 2 on Qwen3-8B it ran 463 tok/s against 527 for the matvec plus
    # the separate peer all-reduce kernel (every CTA of the matvec waits out the flag round trip).
    fused_reduce: bool = False

    def __post_init__(self) -> None:
        super().__post_init__()
        import torch.distributed as dist

        self._dist = dist
        self.embed_vocab = self.full_cfg.vocab
        self.vocab_offset = self.rank * self.cfg.vocab
        g = (self.cfg.vocab + 3) // 4
        self._gather_ps = torch.empty(self.tp, self.batch, g, dtype=torch.float32, device=self.device)
        self._gather_pt = torch.empty(self.tp, self.batch, g, dtype=torch.int32, device=self.device)
        self._peer = None
        if self.peer_allreduce and self.tp > 1:
            from torch2vk_b200.comm import PeerAllReduce

            self._peer = PeerAllReduce(self.group, max_elems=self.batch * self.full_cfg.hidden, device=self.device,
                                       linear_rows=self.full_cfg.hidden if self.fused_reduce else 0)

    def _row_parallel(self, x: torch.Tensor, w, k: int, h: torch.Tensor) -> None:
        """h += the sum over the ranks of x @ W_rank^T: one fused launch at one token, else the local
        matvec (rank 0 adds the residual) and an all-reduce."""
        if self._peer is not None and self._peer.linear(x, w.data, w.kind, k, residual=h, out=h):
            return
        kernels.linear(x, w.data, w.kind, k, residual=h if self.rank == 0 else None, out=h)
        self._all_reduce(h)

    def _all_reduce(self, t: torch.Tensor) -> None:
        if self._peer is not None:
            self._peer(t)  # NCCL for tensors beyond its buffer (prefill)
        else:
            self._dist.all_reduce(t, group=self.group)

    def _layer(self, i: int, b, tokens_per_seq: int, decode: bool) -> None:
        cfg, lw = self.cfg, self.weights.layers[i]
        h = b.h
        full = self.full_cfg
        kernels.linear_multi(h, [(lw.q.data, lw.q.kind), (lw.k.data, lw.k.kind), (lw.v.data, lw.v.kind)],
                             full.hidden, norm_weight=lw.input_norm, eps=cfg.eps, outs=[b.q, b.k, b.v])
        self._attention(i, b, tokens_per_seq, decode)
        # row-parallel o_proj / down_proj: partial sums reduced over the ranks, the residual added once
        self._row_parallel(b.attn, lw.o, cfg.heads * cfg.head_dim, h)
        kernels.linear_swiglu(h, lw.gate.data, lw.up.data, lw.gate.kind, full.hidden, norm_weight=lw.post_norm,
                              eps=cfg.eps, out=b.act)
        self._row_parallel(b.act, lw.down, cfg.intermediate, h)

    def _head(self, x_last: torch.Tensor, b) -> None:
        cfg, w = self.cfg, self.weights
        kernels.lm_head_argmax(x_last, w.lm_head.data, w.lm_head.kind, self.full_cfg.hidden,
                               norm_weight=w.final_norm, eps=cfg.eps, partial_scores=b.ps, partial_tokens=b.pt)
        if self.vocab_offset:
            b.pt.add_(self.vocab_offset)
        self._dist.all_gather_into_tensor(self._gather_ps, b.ps, group=self.group)
        self._dist.all_gather_into_tensor(self._gather_pt, b.pt, group=self.group)
        ps = self._gather_ps.permute(1, 0, 2).reshape(self.batch, -1)
        pt = self._gather_pt.permute(1, 0, 2).reshape(self.batch, -1)
        kernels.token_select(ps.contiguous(), pt.contiguous(), self.eos, next_token=self.next_token, done=self.done)
        kernels.token_store(self.next_token, self.done, self.generated, self.generated_length, self.stopped,
                            token_index_dev=self.token_index, stop_on_eos=bool(self.eos_ids))

    def _embed(self, ids: torch.Tensor, out: torch.Tensor) -> None:
        kernels.embedding(self.weights.embed, self.weights.embed_kind, ids, self.full_cfg.hidden, self.embed_vocab,
                          out=out)


def make_tp_runner(full_cfg: Qwen3Config, full_weights: Qwen3Weights, *, rank: int, tp: int, group=None,
                   **runner_kw) -> TPQwen3Runner:
    cfg = local_config(full_cfg, tp)
    local = shard_weights(full_weights, full_cfg, rank, tp)
    return TPQwen3Runner(cfg=cfg, weights=local, full_cfg=full_cfg, rank=rank, tp=tp, group=group, **runner_kw)

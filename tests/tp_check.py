"""Two-or-more-rank check of tensor-parallel Qwen3 decoding (run under torchrun; used by test_tp_gpu.py).

Every rank builds the same seeded oracle model (oracle/qwen3_ref.py: HF fp32
Qwen3 on the dequantized GGUF blocks; the packed blocks are what the GPU
streams), runs the tensor-parallel runner (prefill + graph-replayed decode),
and rank 0 compares 32 greedy tokens with the oracle's greedy decode and with
the single-GPU runner on the same weights.  Prints
"TP OK first_diff_oracle=<i> first_diff_single=<j> single_vs_oracle=<k> gap_at_single_diff=<g>
ranks_identical=<b> status=<s> min_gap=<g>" (a first_diff of 32 means all 32 tokens agree; the
oracle's top-two logit gap at step j says whether a TP / single-GPU difference sits at a near tie).
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

from test_qwen3_gpu import upload  # noqa: E402

from oracle import qwen3_ref  # noqa: E402
from torch2vk_b200.qwen3 import Qwen3Config, Qwen3Runner  # noqa: E402
from torch2vk_b200.tp import make_tp_runner  # noqa: E402

STEPS = 32


def first_diff(a: torch.Tensor, b: torch.Tensor) -> int:
    ne = (a.cpu() != b.cpu()).nonzero()
    return int(ne[0, -1]) if ne.numel() else a.shape[-1]


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    # 32 Q / 8 KV heads, as the 8B model: heads, KV heads and the 4096-wide projections divide over 2, 4 and 8
    # ranks at Q4_K super-block boundaries
    cfg = Qwen3Config(hidden=1024, layers=4, heads=32, kv_heads=8, head_dim=128, intermediate=4096, vocab=8192)
    pm = qwen3_ref.build(cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab,
                         seed=0, topology="q4_k")
    weights = upload(pm, cfg)
    ids = qwen3_ref.prompt_ids(24, cfg.vocab, seed=0)
    peer = os.environ.get("TP_PEER", "1") == "1"
    fused = os.environ.get("TP_FUSED", "1") == "1"
    tp_runner = make_tp_runner(cfg, weights, rank=rank, tp=world, batch=1, max_seq=128,
                               max_new_tokens=STEPS + 2, peer_allreduce=peer, fused_reduce=fused)
    warm = torch.ones(1, device="cuda")
    dist.all_reduce(warm)  # communicator up before any graph capture
    got = tp_runner.generate(ids.cuda(), STEPS).clone()
    torch.cuda.synchronize()
    everyone = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(everyone, got)
    if rank == 0:
        from torch2vk_b200 import kernels

        single = Qwen3Runner(cfg, weights, batch=1, max_seq=128, max_new_tokens=STEPS + 2)
        ref_single = single.generate(ids.cuda(), STEPS)
        ref_oracle, gaps = qwen3_ref.greedy(pm.hf, ids, STEPS)
        same_across = all(torch.equal(e, got) for e in everyone)
        status = kernels.device_status()
        fd_single = first_diff(got, ref_single)
        gap_at = gaps[fd_single] if fd_single < STEPS else float("inf")
        print(f"TP OK first_diff_oracle={first_diff(got, ref_oracle)} first_diff_single={fd_single} "
              f"single_vs_oracle={first_diff(ref_single, ref_oracle)} gap_at_single_diff={gap_at:.4f} "
              f"ranks_identical={same_across} status={status} min_gap={min(gaps):.4f}", flush=True)
    dist.barrier()
    if tp_runner._peer is not None:
        tp_runner._graph = None
        tp_runner._peer.close()
    del tp_runner
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

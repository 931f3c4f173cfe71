"""Two-or-more-rank check of tensor-parallel Qwen3 decoding (run under torchrun; used by test_tp_gpu.py).

Every rank builds the same seeded weights, runs the TP runner (prefill + graph-replayed decode) and
rank 0 compares the tokens with a single-GPU runner on the same weights.  Prints "TP OK <agree>/<n>".
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from torch2vk_b200.qwen3 import Qwen3Config, Qwen3Runner, random_weights  # noqa: E402
from torch2vk_b200.tp import make_tp_runner  # noqa: E402


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    cfg = Qwen3Config(hidden=1024, layers=4, heads=16, kv_heads=8, head_dim=128, intermediate=3072, vocab=4096)
    weights = random_weights(cfg, seed=3, device=f"cuda:{local}", lm_head_kind="q6_k", topology="q4_k", std=0.05)
    prompt = torch.randint(0, cfg.vocab, (1, 24), generator=torch.Generator().manual_seed(5)).cuda()
    steps = 16
    peer = os.environ.get("TP_PEER", "1") == "1"
    tp_runner = make_tp_runner(cfg, weights, rank=rank, tp=world, batch=1, max_seq=128, max_new_tokens=steps + 2,
                               peer_allreduce=peer)
    warm = torch.ones(1, device="cuda")
    dist.all_reduce(warm)  # communicator up before any graph capture
    got = tp_runner.generate(prompt, steps).clone()
    torch.cuda.synchronize()
    everyone = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(everyone, got)
    if rank == 0:
        single = Qwen3Runner(cfg, weights, batch=1, max_seq=128, max_new_tokens=steps + 2)
        ref = single.generate(prompt, steps)
        same_across = all(torch.equal(e, got) for e in everyone)
        agree = int((ref == got).sum())
        first = int((ref[0] != got[0]).nonzero()[0]) if agree < steps else steps
        from torch2vk_b200 import kernels

        status = kernels.device_status()
        print(f"TP OK {agree}/{steps} first_diff={first} ranks_identical={same_across} status={status}", flush=True)
        if not same_across or first < 8:
            print("TP MISMATCH", ref.tolist(), got.tolist(), flush=True)
    dist.barrier()
    if tp_runner._peer is not None:
        tp_runner._graph = None
        tp_runner._peer.close()
    del tp_runner
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

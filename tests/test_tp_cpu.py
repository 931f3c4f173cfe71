"""Tensor-parallel sharding on CPU: two gloo ranks check that the K-split (row-parallel) and row-split
(column-parallel) cuts of packed GGUF weights, summed / concatenated over ranks with the same
collectives the GPU runner uses, reproduce the full oracle matvec, and that the vocab-split argmax
with global token ids picks the full argmax (lowest id on ties)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle
        from torch2vk_b200.qwen3 import QWeight
        from torch2vk_b200.tp import shard_k, shard_rows

        rng = np.random.default_rng(0)
        n, k = 64, 1024
        errs = []
        for kind in ("q4_k", "q6_k", "q8_0"):
            w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
            packed = oracle.quantize(w, kind)
            phys = torch.from_numpy(oracle.gguf_physical(packed, kind))
            x = rng.standard_normal((2, k)).astype(np.float16)
            full = oracle.matvec(packed, kind, x)
            # row-parallel: each rank's K slice, summed by all_reduce
            part = shard_k(QWeight(phys, kind), k, rank, world)
            kk = k // world
            xs = x[:, rank * kk:(rank + 1) * kk]
            y = torch.from_numpy(oracle.matvec(part.data.view(torch.uint8).numpy(), kind, xs).astype(np.float64))
            dist.all_reduce(y)
            errs.append(float(np.abs(y.numpy() - full).max()))
            # column-parallel: each rank's rows, concatenated by all_gather
            rows = shard_rows(QWeight(phys, kind), rank, world)
            yr = torch.from_numpy(oracle.matvec(rows.data.view(torch.uint8).numpy(), kind, x).astype(np.float64))
            parts = [torch.empty_like(yr) for _ in range(world)]
            dist.all_gather(parts, yr)
            errs.append(float(np.abs(torch.cat(parts, dim=1).numpy() - full).max()))
        # vocab-split argmax with global ids: gathered partial maxima -> global argmax, lowest id on ties
        scores = rng.standard_normal(400).astype(np.float32)
        scores[17] = scores[311] = 10.0
        v = len(scores) // world
        local = scores[rank * v:(rank + 1) * v]
        best = torch.tensor([float(local.max()), float(rank * v + int(np.argmax(local)))], dtype=torch.float64)
        allb = [torch.empty_like(best) for _ in range(world)]
        dist.all_gather(allb, best)
        cand = sorted(((-float(b[0]), int(b[1])) for b in allb))
        q.put((rank, max(errs), cand[0][1]))
    finally:
        dist.destroy_process_group()


def test_tp_sharding_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, tok in results:
        assert err < 1e-5, (rank, err)  # the oracle returns float32 sums
        assert tok == 17

"""Tensor parallelism on real GPUs (needs >= 2): TP=2 greedy tokens vs the single-GPU runner.

The bound: fp16 all-reduces sum the row-parallel partials in a different
order than one GPU does, so tokens may flip only at near-ties; the first 8
tokens must agree and every rank must hold the same tokens.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("peer", ["1", "0"])
def test_tp2_matches_single_gpu(peer):
    """peer=1: decode all-reduces over NVLink peer memory; peer=0: NCCL all-reduce."""
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={29531 + int(peer)}",
           str(REPO / "tests" / "tp_check.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TP_PEER=peer)
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=360)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    line = next(ln for ln in out.splitlines() if ln.startswith("TP OK"))
    assert "ranks_identical=True" in line and "status=0" in line, line
    first = int(line.split("first_diff=")[1].split()[0])
    assert first >= 8, out[-2000:]

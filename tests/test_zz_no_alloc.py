"""t2c_attn_decode_static: decode attention for callers that cannot allocate.

Some hosts own every device allocation themselves (fixed-budget serving
executors, runtimes that plan all memory up front) and do not let a plugin
call cudaMalloc, so they cannot hand t2c_attn_decode a workspace.  This entry
point keeps the split-K partials in a fixed 16 MiB array inside the library.

The test calls both entry points through the C ABI on the same inputs and
checks that the outputs agree within the tolerance the decode-attention tests
use, on two calls in a row (the second reuses the scratch the first one left
behind), and that an oversized request is refused.  The file is named so that
pytest collects it last.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(name: str, q, kc, vc, out, positions, B, NH, NK, D, S, splits, workspace=None):
    from torch2vk_b200 import _lib, kernels

    cb, cs, ch = kernels.cache_strides(kc, "token_major")
    args = [_lib.ptr(q), _lib.ptr(kc), _lib.ptr(vc), _lib.ptr(out), _lib.ptr(positions), B, NH, NK, D, S, cb, cs, ch,
            splits]
    if name == "t2c_attn_decode":
        args += [_lib.ptr(workspace), workspace.numel() if workspace is not None else 0]
    _lib.lib().call(name, *args, _lib.stream_ptr())


def _close(got: torch.Tensor, ref: torch.Tensor, rel: float = 4e-3, abs_: float = 2e-3) -> None:
    err = (got.float() - ref.float()).abs()
    assert bool((err <= rel * ref.float().abs() + abs_).all()), f"max err {float(err.max())}"


def test_static_scratch_matches_workspace_entry_point_twice():
    torch.manual_seed(11)
    B, NH, NK, D, S = 4, 32, 8, 128, 1500
    kc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    vc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    for call, (splits, lens) in enumerate([(12, [1, 700, 1499, 64]), (24, [1500, 3, 999, 1200])]):
        q = torch.randn(B, NH * D, device="cuda", dtype=torch.float16)
        positions = torch.tensor([n - 1 for n in lens], device="cuda", dtype=torch.int32)
        workspace = torch.empty(B * NH * splits * (D + 2), device="cuda", dtype=torch.float32)
        ref = torch.empty_like(q)
        got = torch.empty_like(q)
        _call("t2c_attn_decode", q, kc, vc, ref, positions, B, NH, NK, D, S, splits, workspace)
        _call("t2c_attn_decode_static", q, kc, vc, got, positions, B, NH, NK, D, S, splits)
        torch.cuda.synchronize()
        _close(got, ref)
        assert torch.isfinite(got.float()).all(), f"call {call}: non-finite output"


def test_static_scratch_refuses_oversized_requests():
    from torch2vk_b200 import _lib

    B, NH, NK, D, S = 64, 32, 8, 128, 4096
    q = torch.zeros(B, NH * D, device="cuda", dtype=torch.float16)
    kc = torch.zeros(1, 1, NK, D, device="cuda", dtype=torch.float16)
    positions = torch.zeros(B, device="cuda", dtype=torch.int32)
    with pytest.raises(_lib.T2CError) as info:
        _call("t2c_attn_decode_static", q, kc, kc, q, positions, B, NH, NK, D, S, 64)
    assert info.value.status == 5  # T2C_ESCRATCH

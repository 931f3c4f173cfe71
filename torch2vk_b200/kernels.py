"""Tensor-level wrappers over the C ABI (torch tensors in, torch tensors out).

These are thin: validate dtypes/shapes on the host, pass raw device pointers
and the current CUDA stream to libt2c_sm100.so, and raise on a non-zero status.
Weights are the GGUF packed tensors in the reference's physical dtypes
(Q4_K: uint32 [N, K/256*36]; Q6_K: uint16 [N, K/256*105]; Q8_0: uint16
[N, K/32*17]); any byte-identical view (uint8) is accepted too.
"""

from __future__ import annotations

import torch

from torch2vk_b200 import _lib
from torch2vk_b200._lib import Q4_K, Q6_K, Q8_0, WTYPE_BY_NAME

BLOCK = {Q4_K: (256, 144), Q6_K: (256, 210), Q8_0: (32, 34)}
PHYSICAL_DTYPE = {Q4_K: torch.uint32, Q6_K: torch.uint16, Q8_0: torch.uint16}


def wtype_of(kind: str | int) -> int:
    return WTYPE_BY_NAME[kind] if isinstance(kind, str) else int(kind)


def row_bytes(wtype: int, k: int) -> int:
    block, nbytes = BLOCK[wtype]
    if k % block:
        raise ValueError(f"K={k} is not a multiple of {block} for weight type {wtype}")
    return k // block * nbytes


def _check_weight(w: torch.Tensor, wtype: int, k: int) -> int:
    if not w.is_cuda or not w.is_contiguous():
        raise ValueError("weight must be a contiguous CUDA tensor")
    rb = row_bytes(wtype, k)
    total = w.numel() * w.element_size()
    if total % rb:
        raise ValueError(f"weight has {total} bytes, not a whole number of {rb}-byte rows")
    return total // rb


def _check_x(x: torch.Tensor, k: int) -> int:
    if x.dtype != torch.float16 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous CUDA float16 tensor")
    if x.shape[-1] != k:
        raise ValueError(f"x last dim {x.shape[-1]} != K {k}")
    return x.numel() // k


def linear(x: torch.Tensor, w: torch.Tensor, kind: str | int, k: int, *, residual: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ deq(W)^T (+ residual); x fp16 [..., K] -> y fp16 [..., N]."""
    wtype = wtype_of(kind)
    n = _check_weight(w, wtype, k)
    m = _check_x(x, k)
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=torch.float16, device=x.device)
    if residual is not None and (residual.dtype != torch.float16 or residual.numel() != m * n):
        raise ValueError("residual must be float16 with M*N elements")
    _lib.lib().call("t2c_linear", wtype, _lib.ptr(x), _lib.ptr(w), _lib.ptr(residual), _lib.ptr(out), m, n, k,
                    _lib.stream_ptr())
    return out


def linear_multi(x: torch.Tensor, weights: list[tuple[torch.Tensor, str | int]], k: int, *,
                 norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                 residuals: list[torch.Tensor | None] | None = None,
                 outs: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """One x, up to three weights (fused QKV / gate-up); optional fused RMSNorm prologue."""
    m = _check_x(x, k)
    wtypes, wptrs, ns = [], [], []
    for w, kind in weights:
        wt = wtype_of(kind)
        wtypes.append(wt)
        wptrs.append(_lib.ptr(w))
        ns.append(_check_weight(w, wt, k))
    if outs is None:
        outs = [torch.empty(*x.shape[:-1], n, dtype=torch.float16, device=x.device) for n in ns]
    res = residuals or [None] * len(weights)
    if norm_weight is not None and (norm_weight.dtype != torch.float32 or norm_weight.numel() != k):
        raise ValueError("norm_weight must be float32 [K]")
    _lib.lib().call(
        "t2c_linear_multi", len(weights), _lib.int_array(wtypes), _lib.ptr_array(wptrs),
        _lib.ptr_array([_lib.ptr(o) for o in outs]), _lib.ptr_array([_lib.ptr(r) for r in res]),
        _lib.i64_array(ns), _lib.ptr(x), _lib.ptr(norm_weight), float(eps), m, k, _lib.stream_ptr())
    return outs


def linear_swiglu(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, kind: str | int, k: int, *,
                  norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """y = silu(x Wg^T) * (x Wu^T) with optional fused RMSNorm prologue."""
    wtype = wtype_of(kind)
    n = _check_weight(w_gate, wtype, k)
    if _check_weight(w_up, wtype, k) != n:
        raise ValueError("gate and up must have the same number of rows")
    m = _check_x(x, k)
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=torch.float16, device=x.device)
    _lib.lib().call("t2c_linear_swiglu", wtype, _lib.ptr(x), _lib.ptr(w_gate), _lib.ptr(w_up), _lib.ptr(out),
                    _lib.ptr(norm_weight), float(eps), m, n, k, _lib.stream_ptr())
    return out


def quantize(x: torch.Tensor, kind: str | int) -> torch.Tensor:
    """fp32 [R, K] -> packed GGUF blocks (physical dtype of the reference layout)."""
    wtype = wtype_of(kind)
    if x.dtype != torch.float32 or x.dim() != 2 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("quantize expects a contiguous CUDA float32 [R, K] tensor")
    r, k = x.shape
    rb = row_bytes(wtype, k)
    out = torch.empty(r, rb, dtype=torch.uint8, device=x.device)
    _lib.lib().call("t2c_quantize", wtype, _lib.ptr(x), _lib.ptr(out), r, k, _lib.stream_ptr())
    return out.view(PHYSICAL_DTYPE[wtype])


def dequantize(w: torch.Tensor, kind: str | int, k: int) -> torch.Tensor:
    wtype = wtype_of(kind)
    r = _check_weight(w, wtype, k)
    out = torch.empty(r, k, dtype=torch.float32, device=w.device)
    _lib.lib().call("t2c_dequantize", wtype, _lib.ptr(w), _lib.ptr(out), r, k, _lib.stream_ptr())
    return out

"""Tensor-level wrappers over the C ABI (torch tensors in, torch tensors out).

These are thin: validate dtypes/shapes on the host, pass raw device pointers
and the current CUDA stream to libt2c_sm100.so, and raise on a non-zero status.
Weights are the GGUF packed tensors in the reference's physical dtypes
(Q4_K: uint32 [N, K/256*36]; Q6_K: uint16 [N, K/256*105]; Q8_0: uint16
[N, K/32*17]); any byte-identical view (uint8) is accepted too.
"""

from __future__ import annotations

import ctypes

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


def _fused_norm_ok(m: int, k: int, kinds) -> bool:
    """Whether the kernels that serve M tokens fuse the RMSNorm prologue: the decode matvecs (M <= 4)
    and the batched Q4_K kernel do, the tcgen05 GEMM does not.  The batched kernel serves Q4_K at
    5..16 tokens when K <= 8192, and at 5..8 tokens for any K (qlinear.cu, batched_kernel_serves)."""
    batched = 4 < m <= 16 and (k <= 8192 or m <= 8)
    return m <= 4 or (batched and all(wtype_of(kd) == wtype_of("q4_k") for kd in kinds))


def linear_multi(x: torch.Tensor, weights: list[tuple[torch.Tensor, str | int]], k: int, *,
                 norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                 residuals: list[torch.Tensor | None] | None = None,
                 outs: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """One x, up to three weights (fused QKV / gate-up); optional fused RMSNorm prologue."""
    m = _check_x(x, k)
    if norm_weight is not None and not _fused_norm_ok(m, k, [kind for _, kind in weights]):
        # the tensor-core GEMM reads x as it is: normalize first (torch-allocated temporary)
        x, norm_weight = rms_norm(x, norm_weight, eps), None
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
    if norm_weight is not None and not _fused_norm_ok(m, k, [kind]):
        x, norm_weight = rms_norm(x, norm_weight, eps), None
    _lib.lib().call("t2c_linear_swiglu", wtype, _lib.ptr(x), _lib.ptr(w_gate), _lib.ptr(w_up), _lib.ptr(out),
                    _lib.ptr(norm_weight), float(eps), m, n, k, _lib.stream_ptr())
    return out


def quantize(x: torch.Tensor, kind: str | int, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 [R, K] -> packed GGUF blocks (physical dtype of the reference layout)."""
    wtype = wtype_of(kind)
    if x.dtype != torch.float32 or x.dim() != 2 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("quantize expects a contiguous CUDA float32 [R, K] tensor")
    r, k = x.shape
    rb = row_bytes(wtype, k)
    if out is not None:
        if not out.is_contiguous() or out.numel() * out.element_size() != r * rb:
            raise ValueError(f"out must be contiguous with {r * rb} bytes")
        _lib.lib().call("t2c_quantize", wtype, _lib.ptr(x), _lib.ptr(out), r, k, _lib.stream_ptr())
        return out
    out = torch.empty(r, rb, dtype=torch.uint8, device=x.device)
    _lib.lib().call("t2c_quantize", wtype, _lib.ptr(x), _lib.ptr(out), r, k, _lib.stream_ptr())
    return out.view(PHYSICAL_DTYPE[wtype])


def dequantize(w: torch.Tensor, kind: str | int, k: int) -> torch.Tensor:
    wtype = wtype_of(kind)
    r = _check_weight(w, wtype, k)
    out = torch.empty(r, k, dtype=torch.float32, device=w.device)
    _lib.lib().call("t2c_dequantize", wtype, _lib.ptr(w), _lib.ptr(out), r, k, _lib.stream_ptr())
    return out


# ---------------------------------------------------------------- decode ops
def _check(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor")


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over the last dim: fp16 x, fp32 w."""
    _check(x, torch.float16, "x")
    _check(w, torch.float32, "w")
    cols = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    _lib.lib().call("t2c_rms_norm", _lib.ptr(x), _lib.ptr(w), _lib.ptr(out), x.numel() // cols, cols, float(eps),
                    _lib.stream_ptr())
    return out


def cache_strides(cache: torch.Tensor, layout: str) -> tuple[int, int, int]:
    """(batch, position, head) element strides of a KV cache tensor.

    layout "token_major": [B, S, NK, D]; "head_major": [B, NK, S, D].
    """
    if layout == "token_major":
        return cache.stride(0), cache.stride(1), cache.stride(2)
    if layout == "head_major":
        return cache.stride(0), cache.stride(2), cache.stride(1)
    raise ValueError(layout)


def qk_norm_rope_cache(q_in: torch.Tensor, k_in: torch.Tensor, v_in: torch.Tensor, q_w: torch.Tensor,
                       k_w: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, positions: torch.Tensor,
                       inv_freq: torch.Tensor, *, batch: int, tokens: int, n_heads: int, n_kv: int, head_dim: int,
                       layout: str = "token_major", eps: float = 1e-6,
                       q_out: torch.Tensor | None = None) -> torch.Tensor:
    """q/k RMSNorm + RoPE; rotated k and raw v written into the caches at positions[b] + t."""
    for t, n in ((q_in, "q_in"), (k_in, "k_in"), (v_in, "v_in")):
        _check(t, torch.float16, n)
    _check(positions, torch.int32, "positions")
    _check(inv_freq, torch.float32, "inv_freq")
    q_out = torch.empty_like(q_in) if q_out is None else q_out
    cb, cs, ch = cache_strides(k_cache, layout)
    _lib.lib().call("t2c_qk_norm_rope_cache", _lib.ptr(q_in), _lib.ptr(k_in), _lib.ptr(v_in), _lib.ptr(q_w),
                    _lib.ptr(k_w), _lib.ptr(q_out), _lib.ptr(k_cache), _lib.ptr(v_cache), _lib.ptr(positions),
                    batch, tokens, n_heads, n_kv, head_dim, cb, cs, ch, _lib.ptr(inv_freq), float(eps),
                    _lib.stream_ptr())
    return q_out


def attn_decode_workspace_floats(batch: int, n_heads: int, head_dim: int, splits: int) -> int:
    return batch * n_heads * splits * (head_dim + 2) if splits > 1 else 0


def attn_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, positions: torch.Tensor, *,
                batch: int, n_heads: int, n_kv: int, head_dim: int, max_len: int, splits: int = 1,
                layout: str = "token_major", workspace: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """One query token per batch row against cache positions 0..positions[b]."""
    _check(q, torch.float16, "q")
    out = torch.empty_like(q) if out is None else out
    need = attn_decode_workspace_floats(batch, n_heads, head_dim, splits)
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.float32, device=q.device)
    cb, cs, ch = cache_strides(k_cache, layout)
    _lib.lib().call("t2c_attn_decode", _lib.ptr(q), _lib.ptr(k_cache), _lib.ptr(v_cache), _lib.ptr(out),
                    _lib.ptr(positions), batch, n_heads, n_kv, head_dim, max_len, cb, cs, ch, splits,
                    _lib.ptr(workspace), workspace.numel() if workspace is not None else 0, _lib.stream_ptr())
    return out


def attn_decode_paged(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor, positions: torch.Tensor,
                      block_table: torch.Tensor, *, batch: int, n_heads: int, n_kv: int, head_dim: int,
                      splits: int = 1, workspace: torch.Tensor | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """attn_decode over a paged cache: pages [num_pages, page_size, n_kv, head_dim] fp16, block_table
    [sequences, pages_per_seq] int32 (row b = sequence b's physical pages)."""
    _check(q, torch.float16, "q")
    _check(positions, torch.int32, "positions")
    _check(block_table, torch.int32, "block_table")
    if k_pages.shape != v_pages.shape or k_pages.dim() != 4 or k_pages.dtype != torch.float16:
        raise ValueError("k_pages / v_pages must be float16 [num_pages, page_size, n_kv, head_dim]")
    out = torch.empty_like(q) if out is None else out
    need = attn_decode_workspace_floats(batch, n_heads, head_dim, splits)
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.float32, device=q.device)
    ps, rs, hs, _ = k_pages.stride()
    _lib.lib().call("t2c_attn_decode_paged", _lib.ptr(q), _lib.ptr(k_pages), _lib.ptr(v_pages), _lib.ptr(out),
                    _lib.ptr(positions), _lib.ptr(block_table), block_table.stride(0), k_pages.shape[0],
                    k_pages.shape[1], ps, rs, hs, batch, n_heads, n_kv, head_dim, splits, _lib.ptr(workspace),
                    workspace.numel() if workspace is not None else 0, _lib.stream_ptr())
    return out


def kv_cache_write_paged(pages: torch.Tensor, src: torch.Tensor, positions: torch.Tensor, block_table: torch.Tensor,
                         *, batch: int, tokens: int, n_kv: int, head_dim: int) -> None:
    """Writes src [batch, tokens, n_kv * head_dim] (row views fine) at positions[b] .. + tokens - 1 of each
    sequence's pages."""
    _check(positions, torch.int32, "positions")
    _check(block_table, torch.int32, "block_table")
    if src.dtype != torch.float16 or src.stride(-1) != 1:
        raise ValueError("src must be float16 with unit last stride")
    s3 = src.view(batch, tokens, -1) if src.dim() != 3 else src
    ps, rs, hs, _ = pages.stride()
    _lib.lib().call("t2c_kv_cache_write_paged", _lib.ptr(pages), _lib.ptr(s3), s3.stride(0), s3.stride(1),
                    _lib.ptr(positions), _lib.ptr(block_table), block_table.stride(0), pages.shape[0], pages.shape[1],
                    ps, rs, hs, batch, tokens, n_kv, head_dim, _lib.stream_ptr())


def attn_decode_fused_workspace(batch: int, n_heads: int, n_kv: int, head_dim: int, splits: int,
                                device: torch.device | str = "cuda") -> torch.Tensor | None:
    """Zeroed workspace (split partials + arrival counters) for attn_decode_fused, or None for one split."""
    n = int(_lib.lib().raw("t2c_attn_decode_fused_workspace")(batch, n_heads, n_kv, head_dim, splits))
    return torch.zeros(n, dtype=torch.float32, device=device) if n else None


def attn_decode_fused(q_in: torch.Tensor, k_in: torch.Tensor, v_in: torch.Tensor, q_w: torch.Tensor,
                      k_w: torch.Tensor, inv_freq: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      positions: torch.Tensor, *, batch: int, n_heads: int, n_kv: int, head_dim: int, splits: int,
                      workspace: torch.Tensor | None, layout: str = "token_major", eps: float = 1e-6,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """q/k norm + RoPE, KV write at positions[b], attention over 0..positions[b], one launch (T = 1).

    q_in [B, NH*D], k_in / v_in [B, NK*D] (row views of the QKV outputs are fine: batch stride taken
    from stride(0)); workspace from attn_decode_fused_workspace when splits > 1.
    """
    for t, n in ((q_in, "q_in"), (k_in, "k_in"), (v_in, "v_in")):
        if t.dtype != torch.float16 or not t.is_cuda or t.stride(-1) != 1:
            raise ValueError(f"{n} must be a CUDA float16 tensor with unit last stride")
    _check(positions, torch.int32, "positions")
    out = torch.empty(batch, n_heads * head_dim, dtype=torch.float16, device=q_in.device) if out is None else out
    cb, cs, ch = cache_strides(k_cache, layout)
    max_len = k_cache.shape[1] if layout == "token_major" else k_cache.shape[2]
    if v_cache.shape != k_cache.shape or k_cache.dtype != torch.float16:
        raise ValueError("k_cache / v_cache must be float16 tensors of one shape")
    _lib.lib().call("t2c_attn_decode_fused", _lib.ptr(q_in), _lib.ptr(k_in), _lib.ptr(v_in), q_in.stride(0),
                    k_in.stride(0), v_in.stride(0), _lib.ptr(q_w), _lib.ptr(k_w), _lib.ptr(inv_freq), float(eps),
                    _lib.ptr(k_cache), _lib.ptr(v_cache), cb, cs, ch, _lib.ptr(out), out.stride(0),
                    _lib.ptr(positions), batch, n_heads, n_kv, head_dim, max_len, splits, _lib.ptr(workspace),
                    workspace.numel() if workspace is not None else 0, _lib.stream_ptr())
    return out


def attn_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, positions: torch.Tensor, *,
                 batch: int, tokens: int, n_heads: int, n_kv: int, head_dim: int, layout: str = "token_major",
                 q_layout: str = "token_major", out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of `tokens` new queries (already cached) over positions 0..positions[b]+t.

    q / out are token-major [B, T, NH, D] or, with q_layout="head_major", [B, NH, T, D].
    """
    _check(q, torch.float16, "q")
    out = torch.empty_like(q) if out is None else out
    cb, cs, ch = cache_strides(k_cache, layout)
    D = head_dim
    if q_layout == "token_major":
        qs = (tokens * n_heads * D, n_heads * D, D)
    else:
        qs = (n_heads * tokens * D, D, tokens * D)
    _lib.lib().call("t2c_attn_prefill", _lib.ptr(q), _lib.ptr(k_cache), _lib.ptr(v_cache), _lib.ptr(out),
                    _lib.ptr(positions), batch, tokens, n_heads, n_kv, head_dim, cb, cs, ch, *qs, *qs,
                    _lib.stream_ptr())
    return out


def embedding(weight: torch.Tensor, kind: str | int, ids: torch.Tensor, hidden: int, vocab: int,
              out: torch.Tensor | None = None) -> torch.Tensor:
    _check(ids, torch.int64, "ids")
    wtype = wtype_of(kind)
    out = torch.empty(*ids.shape, hidden, dtype=torch.float16, device=ids.device) if out is None else out
    _lib.lib().call("t2c_embedding", wtype, _lib.ptr(weight), _lib.ptr(ids), _lib.ptr(out), ids.numel(), vocab,
                    hidden, _lib.stream_ptr())
    return out


def add(x: torch.Tensor, r: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    _lib.lib().call("t2c_add", _lib.ptr(x), _lib.ptr(r), _lib.ptr(out), x.numel(), _lib.stream_ptr())
    return out


def swiglu(g: torch.Tensor, u: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(g) if out is None else out
    _lib.lib().call("t2c_swiglu", _lib.ptr(g), _lib.ptr(u), _lib.ptr(out), g.numel(), _lib.stream_ptr())
    return out


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor, kind: str | int, k: int, *,
                   norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                   partial_scores: torch.Tensor | None = None,
                   partial_tokens: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-4-row best (score, token) partials [M, ceil(N/4)] of x @ deq(W)^T."""
    wtype = wtype_of(kind)
    n = _check_weight(w, wtype, k)
    m = _check_x(x, k)
    g = (n + 3) // 4
    if norm_weight is not None and m > 4:
        # the tensor-core GEMM for M > 4 reads x as it is: normalize first (torch-allocated temporary)
        x, norm_weight = rms_norm(x, norm_weight, eps), None
    if partial_scores is None:
        partial_scores = torch.empty(m, g, dtype=torch.float32, device=x.device)
        partial_tokens = torch.empty(m, g, dtype=torch.int32, device=x.device)
    _lib.lib().call("t2c_lm_head_argmax", wtype, _lib.ptr(x), _lib.ptr(w), _lib.ptr(partial_scores),
                    _lib.ptr(partial_tokens), _lib.ptr(norm_weight), float(eps), m, n, k, _lib.stream_ptr())
    return partial_scores, partial_tokens


def token_select(partial_scores: torch.Tensor, partial_tokens: torch.Tensor, eos_ids: torch.Tensor, *,
                 next_token: torch.Tensor | None = None,
                 done: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    m, g = partial_scores.shape
    if next_token is None:
        next_token = torch.empty(m, dtype=torch.int64, device=partial_scores.device)
        done = torch.empty(m, dtype=torch.int32, device=partial_scores.device)
    _lib.lib().call("t2c_token_select", _lib.ptr(partial_scores), _lib.ptr(partial_tokens), m, g, _lib.ptr(eos_ids),
                    eos_ids.numel(), _lib.ptr(next_token), _lib.ptr(done), _lib.stream_ptr())
    return next_token, done


def token_store(next_token: torch.Tensor, done: torch.Tensor, generated: torch.Tensor, generated_length: torch.Tensor,
                stopped: torch.Tensor, *, token_index: int = 0, token_index_dev: torch.Tensor | None = None,
                stop_on_eos: bool = True) -> None:
    b, cap = generated.shape
    _lib.lib().call("t2c_token_store", _lib.ptr(next_token), _lib.ptr(done), _lib.ptr(generated),
                    _lib.ptr(generated_length), _lib.ptr(stopped), b, cap, int(token_index),
                    _lib.ptr(token_index_dev), 1 if stop_on_eos else 0, _lib.stream_ptr())


def advance_positions(positions: torch.Tensor, token_index: torch.Tensor | None = None) -> None:
    """positions += 1 (and token_index += 1) on the device, for replayed decode graphs."""
    _check(positions, torch.int32, "positions")
    _lib.lib().call("t2c_advance_positions", _lib.ptr(positions), positions.numel(), _lib.ptr(token_index),
                    _lib.stream_ptr())


def device_status(clear: bool = True) -> int:
    """Status bits (1 << T2C_E*) that kernels reported since the last clear."""
    bits = ctypes.c_uint(0)
    _lib.lib().call("t2c_device_status", ctypes.addressof(bits), 1 if clear else 0, _lib.stream_ptr())
    return int(bits.value)


def _i64x4(values) -> ctypes.Array:
    vals = list(values)
    if len(vals) != 4:
        raise ValueError("expected 4 values")
    return _lib.i64_array(vals)


def copy4d(src: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
    """dst[...] = src[...] for 4-D views (strides taken from the tensors)."""
    if src.shape != dst.shape or src.dim() != 4 or src.element_size() != dst.element_size():
        raise ValueError("copy4d needs equal 4-D shapes and element sizes")
    _lib.lib().call("t2c_copy4d", src.element_size(), _lib.ptr(src), _i64x4(src.stride()), _lib.ptr(dst),
                    _i64x4(dst.stride()), _i64x4(dst.shape), _lib.stream_ptr())
    return dst


EW_OPS = {"add": 0, "mul": 1, "neg": 2, "silu": 3}


def elementwise4d(op: str, a: torch.Tensor, b: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
    """out = op(a[, b]) over 4-D views; size-1 dims of a/b broadcast."""
    if out.dim() != 4 or a.dim() != 4:
        raise ValueError("elementwise4d needs 4-D views")

    def bstrides(t: torch.Tensor) -> list[int]:
        return [0 if t.shape[i] == 1 and out.shape[i] != 1 else t.stride(i) for i in range(4)]

    is_f32 = 1 if out.dtype == torch.float32 else 0
    _lib.lib().call("t2c_elementwise4d", EW_OPS[op], is_f32, _lib.ptr(a), _i64x4(bstrides(a)), _lib.ptr(b),
                    _i64x4(bstrides(b)) if b is not None else None, _lib.ptr(out), _i64x4(out.stride()),
                    _i64x4(out.shape), _lib.stream_ptr())
    return out


def rope_table(cos_out: torch.Tensor, sin_out: torch.Tensor, *, theta: float, start_position: int,
               attention_scaling: float = 1.0, start_position_dev: torch.Tensor | None = None) -> None:
    """cos / sin [B, T, D] (fp16, or fp32 for the output-f32 variant) at positions start_position + t;
    with start_position_dev (int64 [1] on the GPU) the start is read from device memory instead."""
    b, t, d = cos_out.shape
    if cos_out.dtype != sin_out.dtype or cos_out.dtype not in (torch.float16, torch.float32):
        raise ValueError("cos / sin must both be float16 or both float32")
    if start_position_dev is not None:
        _check(start_position_dev, torch.int64, "start_position_dev")
        _lib.lib().call("t2c_rope_table_dev", _lib.ptr(cos_out), _lib.ptr(sin_out), b, t, d, float(theta),
                        _lib.ptr(start_position_dev), float(attention_scaling),
                        1 if cos_out.dtype == torch.float32 else 0, _lib.stream_ptr())
        return
    name = "t2c_rope_table_f32" if cos_out.dtype == torch.float32 else "t2c_rope_table"
    _lib.lib().call(name, _lib.ptr(cos_out), _lib.ptr(sin_out), b, t, d, float(theta), int(start_position),
                    float(attention_scaling), _lib.stream_ptr())


def rms_norm_rope(x: torch.Tensor, w: torch.Tensor, cos_t: torch.Tensor, sin_t: torch.Tensor, out: torch.Tensor, *,
                  out_strides: tuple[int, int, int], eps: float = 1e-6) -> torch.Tensor:
    """x [B, T, G, D] -> rope(rmsnorm(x) * w), out addressed by strides (b, g, t)."""
    b, t, g, d = x.shape
    _lib.lib().call("t2c_rms_norm_rope", _lib.ptr(x), _lib.ptr(w), _lib.ptr(cos_t), _lib.ptr(sin_t), _lib.ptr(out),
                    b, t, g, d, *out_strides, float(eps), _lib.stream_ptr())
    return out


def kv_cache_write(cache: torch.Tensor, src: torch.Tensor, *, cache_strides_bsh: tuple[int, int, int], seq_len: int,
                   src_strides_bth: tuple[int, int, int], batch: int, heads: int, tokens: int, head_dim: int,
                   positions: torch.Tensor | None = None, position: int = 0) -> None:
    _lib.lib().call("t2c_kv_cache_write", _lib.ptr(cache), _lib.ptr(src), _lib.ptr(positions), int(position), batch,
                    heads, tokens, head_dim, seq_len, *cache_strides_bsh, *src_strides_bth, _lib.stream_ptr())


def token_select_chunks(scores: torch.Tensor, tokens: torch.Tensor, chunk_scores: torch.Tensor,
                        chunk_tokens: torch.Tensor) -> None:
    _lib.lib().call("t2c_token_select_chunks", _lib.ptr(scores), _lib.ptr(tokens), scores.numel(),
                    _lib.ptr(chunk_scores), _lib.ptr(chunk_tokens), _lib.stream_ptr())


# ------------------------------------------------------------------ ASR audio encoder
def _q8_rows(w: torch.Tensor, n: int, k: int) -> None:
    nbytes = (k + 31) // 32 * 34
    if w.numel() * w.element_size() != n * nbytes or not w.is_cuda:
        raise ValueError(f"Q8_0 weight must hold {n} rows of {nbytes} bytes on the GPU")


def linear_q8_0_bias(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, n: int, *, gelu: bool = False,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ deq(W)^T + bias (optional GELU): Q8_0 weights, fp16 x [..., K], fp32 bias [N]."""
    k = x.shape[-1]
    if x.dtype != torch.float16 or not x.is_contiguous():
        raise ValueError("x must be contiguous float16")
    _q8_rows(w, n, k)
    if bias is not None:
        _check(bias, torch.float32, "bias")
    m = x.numel() // k
    out = torch.empty(*x.shape[:-1], n, dtype=torch.float16, device=x.device) if out is None else out
    _lib.lib().call("t2c_linear_q8_0_bias", _lib.ptr(x), _lib.ptr(w), _lib.ptr(bias), _lib.ptr(out), m, n, k,
                    1 if gelu else 0, _lib.stream_ptr())
    return out


def conv2d_q8_0(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, co: int, *, kernel: int = 3,
                stride: int = 2, padding: int = 1, gelu: bool = False, channels_last_out: bool = False,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """NCHW fp16 conv2d with Q8_0 weights [Co, ceil(Ci*kernel^2/32) blocks] and fp32 bias (optional GELU);
    output [B, Co, Ho, Wo], or [B, Ho, Wo, Co] with channels_last_out."""
    if x.dtype != torch.float16 or x.dim() != 4 or not x.is_contiguous():
        raise ValueError("x must be a contiguous float16 [B, Ci, H, W] tensor")
    b, ci, hi, wi = x.shape
    _q8_rows(w, co, ci * kernel * kernel)
    ho = (hi + 2 * padding - kernel) // stride + 1
    wo = (wi + 2 * padding - kernel) // stride + 1
    if out is None:
        shape = (b, ho, wo, co) if channels_last_out else (b, co, ho, wo)
        out = torch.empty(*shape, dtype=torch.float16, device=x.device)
    _lib.lib().call("t2c_conv2d_q8_0_nhwc" if channels_last_out else "t2c_conv2d_q8_0", _lib.ptr(x), _lib.ptr(w), _lib.ptr(bias), _lib.ptr(out), b, ci, hi, wi, co,
                    ho, wo, kernel, kernel, stride, stride, padding, padding, 1 if gelu else 0, _lib.stream_ptr())
    return out


def im2col(x: torch.Tensor, *, channels: int, height: int, width: int, strides_bchw: tuple[int, int, int, int],
           batch: int, kernel: int = 3, stride: int = 2, padding: int = 1, kp: int, channels_last: bool = False,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """Columns [batch * Ho * Wo, kp] fp16 of a 2-D convolution over x (fp16, read through element strides
    (b, c, h, w): NCHW, or the [B, H, W, C] rows a GEMM wrote), zero outside the image and past
    channels * kernel^2 columns, K ordered (c, i, j); channels_last: x has unit channel stride (16-byte
    gathers of 8 channels for a 3 x 3 kernel)."""
    if x.dtype != torch.float16 or not x.is_cuda:
        raise ValueError("x must be a float16 CUDA tensor")
    ho = (height + 2 * padding - kernel) // stride + 1
    wo = (width + 2 * padding - kernel) // stride + 1
    rows = batch * ho * wo
    if out is None:
        out = torch.empty(rows, kp, dtype=torch.float16, device=x.device)
    elif out.dtype != torch.float16 or not out.is_contiguous() or out.numel() != rows * kp:
        raise ValueError(f"out must be a contiguous float16 tensor of {rows} x {kp}")
    _lib.lib().call("t2c_im2col_f16", _lib.ptr(x), _lib.ptr(out), batch, channels, height, width, ho, wo, kernel,
                    kernel, stride, stride, padding, padding, kp, _i64x4(strides_bchw), 1 if channels_last else 0,
                    _lib.stream_ptr())
    return out


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5,
               out: torch.Tensor | None = None, *, pad_to: int | None = None) -> torch.Tensor:
    """Row LayerNorm; pad_to: output rows of pad_to columns, the columns past x's written as zeros."""
    cols = x.shape[-1]
    _check(w, torch.float32, "w")
    _check(b, torch.float32, "b")
    if pad_to is not None and pad_to != cols:
        rows = x.numel() // cols
        if out is None:
            out = torch.empty(rows, pad_to, dtype=torch.float16, device=x.device)
        elif out.dtype != torch.float16 or not out.is_contiguous() or out.numel() != rows * pad_to:
            raise ValueError(f"out must be a contiguous float16 tensor of {rows} x {pad_to}")
        _lib.lib().call("t2c_layer_norm_padded", _lib.ptr(x), _lib.ptr(w), _lib.ptr(b), _lib.ptr(out), rows, cols,
                        pad_to, float(eps), _lib.stream_ptr())
        return out
    out = torch.empty_like(x) if out is None else out
    _lib.lib().call("t2c_layer_norm", _lib.ptr(x), _lib.ptr(w), _lib.ptr(b), _lib.ptr(out), x.numel() // cols, cols,
                    float(eps), _lib.stream_ptr())
    return out


def gelu(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    _lib.lib().call("t2c_gelu", _lib.ptr(x), _lib.ptr(out), x.numel(), _lib.stream_ptr())
    return out


def index_rows(x: torch.Tensor, index: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    h = x.shape[-1]
    rows = x.numel() // h
    _check(index, torch.int64, "index")
    out = torch.empty(index.numel(), h, dtype=x.dtype, device=x.device) if out is None else out
    _lib.lib().call("t2c_index_rows", _lib.ptr(x), _lib.ptr(index), _lib.ptr(out), index.numel(), h, rows,
                    _lib.stream_ptr())
    return out


def attn_masked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor, *, scale: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """q [B, H, T, D], k / v [B, H, S, D], additive fp16 mask broadcastable to [B, H, T, S] (unit key stride)."""
    B, H, T, D = q.shape
    S = k.shape[2]
    out = torch.empty(B, H, T, D, dtype=torch.float16, device=q.device) if out is None else out
    m = mask.expand(B, H, T, S)
    if m.stride(3) != 1:
        raise ValueError("mask must have unit stride along keys")

    def st(t):
        return _lib.i64_array([t.stride(0), t.stride(1), t.stride(2)])

    _lib.lib().call("t2c_attn_masked", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(mask), _lib.ptr(out), B, H, T,
                    S, D, st(q), st(k), st(v), st(m), st(out), float(scale), _lib.stream_ptr())
    return out


def attn_masked_gqa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor, *, batch: int,
                    tokens: int, n_heads: int, n_kv: int, head_dim: int, layout: str = "token_major",
                    scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Bidirectional GQA attention under an additive fp16 mask [B, (1,) T, S] (unit key stride).

    layout "token_major": q / out [B, T, NH, D] (row views fine), k / v [B, S, NK, D];
    "head_major": q / out [B, NH, T, D], k / v [B, NK, S, D]."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (mask, "mask")):
        _check(t, torch.float16, n)
    out = torch.empty_like(q) if out is None else out
    if k.stride() != v.stride() or k.shape != v.shape:
        raise ValueError("k and v must have the same shape and strides")
    if mask.stride(-1) != 1 or mask.shape[-2] != tokens:
        raise ValueError("mask must be [B, (1,) T, S] with unit key stride")
    S = mask.shape[-1]
    if layout == "token_major":
        q4, o4 = q.view(batch, tokens, n_heads, head_dim), out.view(batch, tokens, n_heads, head_dim)
        st = lambda t: [t.stride(0), t.stride(1), t.stride(2)]  # noqa: E731
    elif layout == "head_major":
        q4, o4 = q, out
        st = lambda t: [t.stride(0), t.stride(2), t.stride(1)]  # noqa: E731
    else:
        raise ValueError(layout)
    scale = head_dim ** -0.5 if scale is None else scale
    _lib.lib().call("t2c_attn_masked_gqa", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(mask), _lib.ptr(out),
                    batch, tokens, S, n_heads, n_kv, head_dim, _lib.i64_array(st(q4)), _lib.i64_array(st(k)),
                    _lib.i64_array(st(o4)), mask.stride(0) if mask.shape[0] > 1 else 0, mask.stride(-2),
                    float(scale), _lib.stream_ptr())
    return out


# ------------------------------------------------ fp32-activation prefill programs
def _check_f32(t: torch.Tensor, name: str) -> None:
    _check(t, torch.float32, name)


def linear_f32(x: torch.Tensor, w: torch.Tensor, kind: str | int, k: int, *,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """y fp32 [..., N] = x fp32 [..., K] @ deq(W)^T (x rounded to fp16 for the tensor cores)."""
    _check_f32(x, "x")
    if x.shape[-1] != k:
        raise ValueError(f"x last dim {x.shape[-1]} != K {k}")
    wtype = wtype_of(kind)
    n = _check_weight(w, wtype, k)
    m = x.numel() // k
    out = torch.empty(*x.shape[:-1], n, dtype=torch.float32, device=x.device) if out is None else out
    _check_f32(out, "out")
    nbytes = _lib.lib().raw("t2c_linear_f32_scratch_bytes")(m, n, k)
    scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=x.device)
    base = (-scratch.data_ptr()) % 256
    _lib.lib().call("t2c_linear_f32", wtype, _lib.ptr(x), _lib.ptr(w), _lib.ptr(out), m, n, k,
                    scratch.data_ptr() + base, nbytes, _lib.stream_ptr())
    return out


def rms_norm_f32(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 RMSNorm over the last dim (fp32 weight)."""
    _check_f32(x, "x")
    _check_f32(w, "w")
    h = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    _check_f32(out, "out")
    _lib.lib().call("t2c_rms_norm_f32", _lib.ptr(x), _lib.ptr(w), _lib.ptr(out), x.numel() // h, h, float(eps),
                    _lib.stream_ptr())
    return out


def rms_norm_rope_f32(x: torch.Tensor, w: torch.Tensor, cos_t: torch.Tensor, sin_t: torch.Tensor,
                      out: torch.Tensor, *, eps: float = 1e-6) -> torch.Tensor:
    """x fp32 [B, T, G, D] -> rope(rmsnorm(x) * w) [B, T, G, D] in out's dtype (fp32 or fp16)."""
    _check_f32(x, "x")
    _check_f32(w, "w")
    _check(cos_t, torch.float16, "cos")
    _check(sin_t, torch.float16, "sin")
    if out.dtype not in (torch.float32, torch.float16) or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 or float16 tensor")
    B, T, G, D = x.shape
    _lib.lib().call("t2c_rms_norm_rope_f32", _lib.ptr(x), _lib.ptr(w), _lib.ptr(cos_t), _lib.ptr(sin_t), _lib.ptr(out),
                    int(out.dtype == torch.float32), B, T, G, D, float(eps), _lib.stream_ptr())
    return out


def add_f32(x: torch.Tensor, y: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    for t, n in ((x, "x"), (y, "y")):
        _check_f32(t, n)
    out = torch.empty_like(x) if out is None else out
    _lib.lib().call("t2c_binary_f32", 0, _lib.ptr(x), _lib.ptr(y), _lib.ptr(out), x.numel(), _lib.stream_ptr())
    return out


def swiglu_f32(g: torch.Tensor, u: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(g) * u in fp32."""
    for t, n in ((g, "gate"), (u, "up")):
        _check_f32(t, n)
    out = torch.empty_like(g) if out is None else out
    _lib.lib().call("t2c_binary_f32", 1, _lib.ptr(g), _lib.ptr(u), _lib.ptr(out), g.numel(), _lib.stream_ptr())
    return out


_DTYPE_CODE = {torch.float32: _lib.F32, torch.float16: _lib.F16}


def cast(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out = x converted between float32 and float16 (same number of elements)."""
    if x.numel() != out.numel() or not x.is_contiguous() or not out.is_contiguous():
        raise ValueError("cast needs contiguous tensors of equal size")
    _lib.lib().call("t2c_cast", _lib.ptr(x), _DTYPE_CODE[x.dtype], _lib.ptr(out), _DTYPE_CODE[out.dtype], x.numel(),
                    _lib.stream_ptr())
    return out


def slice_last_f32_to_f16(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out [B, 1, H] fp16 = x [B, S, H] fp32 at the last position."""
    _check_f32(x, "x")
    _check(out, torch.float16, "out")
    B, S, H = x.shape
    _lib.lib().call("t2c_slice_last_f32_to_f16", _lib.ptr(x), _lib.ptr(out), B, S, H, _lib.stream_ptr())
    return out


def value_cache_write_f32(src: torch.Tensor, positions: torch.Tensor, caches: list[torch.Tensor]) -> None:
    """fp16 token-major caches [B, S_c, H, D] get src [B, T, H, D] (fp32) at rows positions[t]."""
    _check_f32(src, "src")
    _check(positions, torch.int64, "cache_position")
    B, T, H, D = src.shape
    for c in caches:
        _check(c, torch.float16, "cache")
        if c.shape[0] != B or c.shape[2] != H or c.shape[3] != D:
            raise ValueError(f"cache shape {tuple(c.shape)} does not match src {tuple(src.shape)}")
    _lib.lib().call("t2c_value_cache_write_f32", _lib.ptr(src), _lib.ptr(positions), len(caches),
                    _lib.ptr_array([_lib.ptr(c) for c in caches]), _lib.i64_array([c.shape[1] for c in caches]),
                    B, T, H, D, _lib.stream_ptr())


def fa_mask_opt(mask: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """2-bit codes per (16-row, 64-column) block of the fp16 mask [T, S], written [row_blocks][words]."""
    _check(mask, torch.float16, "mask")
    if out.dtype not in (torch.uint32, torch.int32) or not out.is_contiguous():
        raise ValueError("out must be a contiguous 32-bit tensor")
    T, S = mask.shape
    words, row_blocks = (S + 1023) // 1024, (T + 15) // 16
    if out.numel() < words * row_blocks:
        raise ValueError(f"out holds {out.numel()} words, needs {words * row_blocks}")
    _lib.lib().call("t2c_fa_mask_opt", _lib.ptr(mask), _lib.ptr(out), T, S, words, row_blocks, _lib.stream_ptr())
    return out


def attn_prefill_masked_f32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor,
                            mask_opt: torch.Tensor | None, out: torch.Tensor, *, scale: float) -> torch.Tensor:
    """softmax(q k^T * scale + mask) v; q / out fp32 [B, T, NH, D], k / v fp16 [B, S, NK, D], mask fp16 [T, S]."""
    _check_f32(q, "q")
    _check_f32(out, "out")
    _check(k, torch.float16, "k")
    _check(v, torch.float16, "v")
    _check(mask, torch.float16, "mask")
    B, T, NH, D = q.shape
    S, NK = k.shape[1], k.shape[2]
    words = (S + 1023) // 1024
    if mask_opt is not None and mask_opt.numel() < words * ((T + 15) // 16):
        raise ValueError("mask_opt is smaller than the mask's block grid")
    _lib.lib().call("t2c_attn_prefill_masked_f32", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(mask),
                    _lib.ptr(mask_opt), _lib.ptr(out), B, T, S, NH, NK, D, mask.shape[1], words, float(scale),
                    _lib.stream_ptr())
    return out


def embedding_f32(weight: torch.Tensor, kind: str | int, ids: torch.Tensor, hidden: int, vocab: int,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """out fp32 [..., hidden] = dequantized rows ids of a Q4_K embedding."""
    _check(ids, torch.int64, "ids")
    out = torch.empty(*ids.shape, hidden, dtype=torch.float32, device=ids.device) if out is None else out
    _check_f32(out, "out")
    _lib.lib().call("t2c_embedding_f32", wtype_of(kind), _lib.ptr(weight), _lib.ptr(ids), _lib.ptr(out), ids.numel(),
                    vocab, hidden, _lib.stream_ptr())
    return out


def index_copy_rows(cache: torch.Tensor, index: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """cache [B, T, H][b, index[s]] = src [B, S, H][b, s] (fp16, in place)."""
    _check(cache, torch.float16, "cache")
    _check(src, torch.float16, "src")
    _check(index, torch.int64, "index")
    B, T, H = cache.shape
    S = src.shape[1]
    if src.shape[0] != B or src.shape[2] != H or index.numel() != S:
        raise ValueError(f"index_copy: cache {tuple(cache.shape)} src {tuple(src.shape)} index {index.numel()}")
    _lib.lib().call("t2c_index_copy_rows", _lib.ptr(cache), _lib.ptr(index), _lib.ptr(src), B, T, S, H,
                    _lib.stream_ptr())
    return cache


def embedding_q8_0(weight: torch.Tensor, ids: torch.Tensor, hidden: int, vocab: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """out fp16 [..., hidden] = dequantized Q8_0 rows ids."""
    _check(ids, torch.int64, "ids")
    _check_weight(weight, Q8_0, hidden)
    out = torch.empty(*ids.shape, hidden, dtype=torch.float16, device=ids.device) if out is None else out
    _check(out, torch.float16, "out")
    _lib.lib().call("t2c_embedding_q8_0", _lib.ptr(weight), _lib.ptr(ids), _lib.ptr(out), ids.numel(), vocab, hidden,
                    _lib.stream_ptr())
    return out


EM_OPS = {"pow2": 0, "rsqrt": 1, "add_scalar": 2, "mul_row": 3, "mul_col": 4}


def ew_misc(op: str, a: torch.Tensor, out: torch.Tensor, b: torch.Tensor | None = None, *, H: int = 0,
            scalar: float = 0.0) -> torch.Tensor:
    """Mixed fp16 / fp32 elementwise step (fp32 arithmetic): pow2, rsqrt, add_scalar, mul_row
    (a[i] * b[i // H]) or mul_col (a[i] * b[i % H])."""
    for t in (a, out) + ((b,) if b is not None else ()):
        if t.dtype not in (torch.float16, torch.float32) or not t.is_contiguous() or not t.is_cuda:
            raise ValueError("ew_misc operands must be contiguous CUDA float16 / float32 tensors")
    if out.numel() != a.numel():
        raise ValueError("ew_misc: out and a differ in size")
    f16 = lambda t: int(t is not None and t.dtype == torch.float16)  # noqa: E731
    _lib.lib().call("t2c_ew_misc", EM_OPS[op], _lib.ptr(a), f16(a), _lib.ptr(b), f16(b), _lib.ptr(out), f16(out),
                    a.numel(), int(H), float(scalar), _lib.stream_ptr())
    return out


def row_mean_f32(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[r] = mean over the last dim of fp32 x."""
    _check_f32(x, "x")
    _check_f32(out, "out")
    cols = x.shape[-1]
    if out.numel() != x.numel() // cols:
        raise ValueError("row_mean_f32: out must hold one value per row")
    _lib.lib().call("t2c_row_mean_f32", _lib.ptr(x), _lib.ptr(out), x.numel() // cols, cols, _lib.stream_ptr())
    return out

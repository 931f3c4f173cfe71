"""GPU parity of the quantizers, decoders and quantized linear kernels.

Tier 1 (bit-exact): GPU quantizer bytes == CPU oracle bytes; GPU decoder
floats == oracle decoder floats.  Tier 2 (tolerance): the quantized linear
against the oracle's direct block matvec (double accumulation over the same
fp16 x and the same packed weights).  The tolerance is written below: the
matvec kernels (M <= 4) take the fp16 x as it is (fp32 accumulation, fp16
store), so |err| <= 2e-3 * (|ref| + rms(ref)) is loose for them (the tight
per-output bound is in test_activation_outliers_gpu.py); the tensor-core GEMM
(M > 4) computes on fp16-rounded weights and gets 4e-3.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

KINDS = ["q4_k", "q6_k", "q8_0"]


def _weights(rng: np.random.Generator, n: int, k: int, special: bool = True) -> np.ndarray:
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if special and n >= 8:
        w[0] = 0.0                      # all-zero row
        w[1] = 0.013                    # constant positive row
        w[2, : k // 2] = -0.5           # large negative half
        w[3] = np.abs(w[3])             # all non-negative (min clamps to 0)
        w[4, ::7] = 3.0                 # outliers
        w[5] = w[5] * 1e-7              # tiny values (fp16 subnormal scales)
    return w


def _tol_check(got: np.ndarray, ref: np.ndarray, rel: float = 2e-3) -> None:
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2))) + 1e-30
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bound = rel * (np.abs(ref) + rms)
    worst = np.argmax(err - bound)
    assert np.all(err <= bound), f"max err {err.flat[worst]} > bound {bound.flat[worst]} (ref {ref.flat[worst]})"


def _swiglu_check(got: np.ndarray, g: np.ndarray, u: np.ndarray, rel: float) -> None:
    """silu(g) * u where g and u may each differ from the oracle as a plain GEMM output may (rel times
    |value| + rms), propagated to first order, plus the fp16 rounding of the output."""
    sg = 1.0 / (1.0 + np.exp(-g))
    silu, dsilu = g * sg, sg * (1.0 + g * (1.0 - sg))
    ref = silu * u
    eg = rel * (np.abs(g) + np.sqrt(np.mean(g * g)))
    eu = rel * (np.abs(u) + np.sqrt(np.mean(u * u)))
    bound = np.abs(dsilu * u) * eg + np.abs(silu) * eu + 1e-3 * np.abs(ref) + 1e-6
    err = np.abs(got.astype(np.float64) - ref)
    worst = np.argmax(err - bound)
    assert np.all(err <= bound), f"max err {err.flat[worst]} > bound {bound.flat[worst]} (ref {ref.flat[worst]})"


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("shape", [(64, 256), (37, 1024), (8, 4096)])
def test_quantize_bit_exact(oracle, kind, shape):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(hash((kind, shape)) % 2**32)
    x = _weights(rng, *shape)
    want = oracle.quantize(x, kind)
    got = kernels.quantize(torch.from_numpy(x).cuda(), kind)
    got_bytes = got.view(torch.uint8).cpu().numpy()
    mismatch = np.argwhere(got_bytes != want)
    assert mismatch.size == 0, f"{kind}: {len(mismatch)} bytes differ, first at {mismatch[:3].tolist()}"


@pytest.mark.parametrize("kind", KINDS)
def test_dequantize_bit_exact(oracle, kind):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(7)
    n, k = 48, 1024
    packed = oracle.quantize(_weights(rng, n, k), kind)
    want = oracle.dequantize(packed, kind, k)
    got = kernels.dequantize(torch.from_numpy(packed).cuda(), kind, k).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("m", [1, 2, 3, 4, 8, 11])
@pytest.mark.parametrize("nk", [(256, 1024), (1030, 2048), (96, 3072), (40, 12288)])
def test_linear_parity(oracle, kind, m, nk):
    from torch2vk_b200 import kernels

    n, k = nk
    rng = np.random.default_rng(n * 31 + k + m)
    packed = oracle.quantize(_weights(rng, n, k), kind)
    x = rng.standard_normal((m, k)).astype(np.float16)
    ref = oracle.matvec(packed, kind, x)
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), kind, k)
    # Q4_K, Q8_0, and Q6_K with K a multiple of 2048 or N a multiple of 8, run on the tensor-core GEMM for M > 4,
    # whose operands are fp16 (dequantized weights rounded to fp16, relative 2^-11 each): its bound against the
    # exact double-precision matvec is 4e-3.
    tensor_core = m > 4 and (kind in ("q4_k", "q8_0") or (kind == "q6_k" and (k % 2048 == 0 or n % 8 == 0)))
    _tol_check(y.float().cpu().numpy(), ref, rel=4e-3 if tensor_core else 2e-3)


@pytest.mark.parametrize("kind", ["q4_k", "q6_k"])
def test_linear_residual(oracle, kind):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(3)
    n, k, m = 512, 2048, 1
    packed = oracle.quantize(_weights(rng, n, k), kind)
    x = rng.standard_normal((m, k)).astype(np.float16)
    res = rng.standard_normal((m, n)).astype(np.float16)
    ref = oracle.matvec(packed, kind, x) + res.astype(np.float32)
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), kind, k,
                       residual=torch.from_numpy(res).cuda())
    _tol_check(y.float().cpu().numpy(), ref)


@pytest.mark.parametrize("m,k", [(1, 1024), (16, 2048)])
def test_linear_multi_mixed_types_with_norm(oracle, m, k):
    """QKV with a Q6_K v (LinearNobiasQ4QKQ6VMatvecProgram) and the fused RMSNorm prologue.

    m = 16, K = 2048: the tensor-core GEMM, one launch per weight format (bound 4e-3 as for the GEMM)."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(11)
    specs = [(2048, "q4_k"), (1024, "q4_k"), (1024, "q6_k")]
    packed = [oracle.quantize(_weights(rng, n, k, special=False), kind) for n, kind in specs]
    x = rng.standard_normal((m, k)).astype(np.float16)
    nw = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    xf = x.astype(np.float32)
    xn = xf / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + 1e-6) * nw
    outs = kernels.linear_multi(
        torch.from_numpy(x).cuda(), [(torch.from_numpy(p).cuda(), kind) for p, (_, kind) in zip(packed, specs)], k,
        norm_weight=torch.from_numpy(nw).cuda(), eps=1e-6)
    for out, p, (_, kind) in zip(outs, packed, specs):
        w = oracle.dequantize(p, kind, k).astype(np.float64)
        ref = xn.astype(np.float64) @ w.T
        _tol_check(out.float().cpu().numpy(), ref, rel=4e-3 if m > 4 else 2e-3)


@pytest.mark.parametrize("m", [1, 4])
def test_linear_swiglu(oracle, m):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(5)
    n, k = 3072, 1024
    pg = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
    pu = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
    x = rng.standard_normal((m, k)).astype(np.float16)
    g = oracle.matvec(pg, "q4_k", x).astype(np.float64)
    u = oracle.matvec(pu, "q4_k", x).astype(np.float64)
    ref = g / (1.0 + np.exp(-g)) * u
    y = kernels.linear_swiglu(torch.from_numpy(x).cuda(), torch.from_numpy(pg).cuda(), torch.from_numpy(pu).cuda(),
                              "q4_k", k)
    _tol_check(y.float().cpu().numpy(), ref, rel=4e-3)


def test_linear_rejects_bad_shapes():
    from torch2vk_b200 import _lib, kernels

    x = torch.zeros(1, 300, dtype=torch.float16, device="cuda")
    w = torch.zeros(4, 36, dtype=torch.uint32, device="cuda")
    with pytest.raises(ValueError):
        kernels.linear(x, w, "q4_k", 300)
    with pytest.raises(_lib.T2CError):
        _lib.lib().call("t2c_linear", _lib.Q4_K, _lib.ptr(x), None, None, _lib.ptr(x), 1, 4, 256, _lib.stream_ptr())


@pytest.mark.parametrize("m", [1, 3])
def test_linear_multi_q4k_tensor_core_path(oracle, m):
    """All-Q4_K QKV (the tensor-core kernel) with the fused RMSNorm prologue and ragged row counts."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(17)
    k = 2048
    specs = [2064, 1000, 24]
    packed = [oracle.quantize(_weights(rng, n, k), "q4_k") for n in specs]
    x = rng.standard_normal((m, k)).astype(np.float16)
    nw = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    xf = x.astype(np.float32)
    xn = xf / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + 1e-6) * nw
    outs = kernels.linear_multi(torch.from_numpy(x).cuda(), [(torch.from_numpy(p).cuda(), "q4_k") for p in packed], k,
                                norm_weight=torch.from_numpy(nw).cuda(), eps=1e-6)
    for out, p in zip(outs, packed):
        ref = xn.astype(np.float64) @ oracle.dequantize(p, "q4_k", k).astype(np.float64).T
        _tol_check(out.float().cpu().numpy(), ref)


@pytest.mark.parametrize("m,n,k", [(1, 1030, 768), (3, 96, 1280), (2, 200, 2304)])
def test_q4k_exact_kernel_odd_superblock_counts(oracle, m, n, k):
    """Q4_K with K / 256 odd (no 512-value segments): the exact fp16-x kernel, one pass per token."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(m * 13 + n + k)
    packed = oracle.quantize(_weights(rng, n, k), "q4_k")
    x = rng.standard_normal((m, k)).astype(np.float16)
    ref = oracle.matvec(packed, "q4_k", x)
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), "q4_k", k)
    _tol_check(y.float().cpu().numpy(), ref)


@pytest.mark.parametrize("m,n,k", [(5, 128, 256), (16, 1030, 1024), (64, 384, 4096), (300, 200, 2048),
                                   (33, 96, 12288)])
def test_q4k_gemm_tensor_cores(oracle, m, n, k):
    """M > 4: the tcgen05 GEMM (weights dequantized to fp16 in shared memory, fp32 TMEM accumulators)."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(m * 7 + n + k)
    packed = oracle.quantize(_weights(rng, n, k), "q4_k")
    x = rng.standard_normal((m, k)).astype(np.float16)
    res = rng.standard_normal((m, n)).astype(np.float16)
    w = oracle.dequantize(packed, "q4_k", k).astype(np.float16).astype(np.float64)  # fp16 operands
    ref = x.astype(np.float64) @ w.T + res
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), "q4_k", k,
                       residual=torch.from_numpy(res).cuda())
    _tol_check(y.float().cpu().numpy(), ref, rel=3e-3)


@pytest.mark.parametrize("m,n,k", [(5, 1024, 3072), (64, 200, 1024), (300, 136, 256), (17, 3072, 1280),
                                   (129, 1024, 3072), (40, 1030, 3072)])
def test_q6k_gemm_any_k(oracle, m, n, k):
    """Q6_K on the tcgen05 GEMM for every K % 256 == 0: K % 2048 != 0 rows (not 16-byte multiples) arrive
    through eight-row group maps.  N % 8 != 0 with such K stays on the fp16-x matvec passes."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(m * 5 + n + k)
    packed = oracle.quantize(_weights(rng, n, k), "q6_k")
    x = rng.standard_normal((m, k)).astype(np.float16)
    res = rng.standard_normal((m, n)).astype(np.float16)
    if n % 8 == 0:
        w = oracle.dequantize(packed, "q6_k", k).astype(np.float16).astype(np.float64)  # fp16 operands
        ref = x.astype(np.float64) @ w.T + res
    else:
        ref = oracle.matvec(packed, "q6_k", x).astype(np.float64) + res
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), "q6_k", k,
                       residual=torch.from_numpy(res).cuda())
    _tol_check(y.float().cpu().numpy(), ref, rel=3e-3)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("m", [7, 130])
def test_q4k_gemm_swiglu_and_norm(oracle, m):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(m)
    n, k = 640, 1024
    pg = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
    pu = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
    x = rng.standard_normal((m, k)).astype(np.float16)
    nw = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    xf = x.astype(np.float32)
    xn = (xf / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + 1e-6) * nw).astype(np.float16).astype(np.float64)
    g = xn @ oracle.dequantize(pg, "q4_k", k).astype(np.float16).astype(np.float64).T
    u = xn @ oracle.dequantize(pu, "q4_k", k).astype(np.float16).astype(np.float64).T
    ref = g / (1.0 + np.exp(-g)) * u
    y = kernels.linear_swiglu(torch.from_numpy(x).cuda(), torch.from_numpy(pg).cuda(), torch.from_numpy(pu).cuda(),
                              "q4_k", k, norm_weight=torch.from_numpy(nw).cuda())
    _tol_check(y.float().cpu().numpy(), ref, rel=5e-3)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("m,n,k,swiglu", [(32, 256, 4096, False), (32, 4096, 4096, False), (32, 512, 2048, True),
                                          (48, 300, 12288, False),
                                          # SwiGLU at <= 32 tokens stacks 64 gate rows over 64 up rows in one
                                          # tile: no split (12288 rows), ragged rows with a split, fewer tokens
                                          (20, 12288, 4096, True), (32, 1000, 4096, True), (17, 3000, 2048, True)])
def test_q4k_gemm_cluster_split_k(oracle, m, n, k, swiglu):
    """Small M with few row tiles: K is split over a CTA cluster and reduced through distributed shared memory;
    every CTA of the cluster finishes its share of the token columns."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(n + k + m)
    x = rng.standard_normal((m, k)).astype(np.float16)
    pg = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
    g = x.astype(np.float64) @ oracle.dequantize(pg, "q4_k", k).astype(np.float16).astype(np.float64).T
    if swiglu:
        pu = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
        u = x.astype(np.float64) @ oracle.dequantize(pu, "q4_k", k).astype(np.float16).astype(np.float64).T
        y = kernels.linear_swiglu(torch.from_numpy(x).cuda(), torch.from_numpy(pg).cuda(),
                                  torch.from_numpy(pu).cuda(), "q4_k", k)
        _swiglu_check(y.float().cpu().numpy(), g, u, rel=4e-3)
        assert kernels.device_status() == 0
        return
    else:
        ref = g
        y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(pg).cuda(), "q4_k", k)
    _tol_check(y.float().cpu().numpy(), ref, rel=4e-3)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("m,n,k", [(32, 4096, 4096), (24, 1030, 12288), (40, 1000, 2048)])
def test_q4k_gemm_split_k_residual(oracle, m, n, k):
    """The residual epilogue after the cluster split-K sum (o_proj / down_proj at batch-32 decode shapes)."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(m * n + k)
    x = rng.standard_normal((m, k)).astype(np.float16)
    packed = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
    r = rng.standard_normal((m, n)).astype(np.float16)
    ref = x.astype(np.float64) @ oracle.dequantize(packed, "q4_k", k).astype(np.float16).astype(np.float64).T
    ref = ref + r.astype(np.float64)
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), "q4_k", k,
                       residual=torch.from_numpy(r).cuda())
    _tol_check(y.float().cpu().numpy(), ref, rel=4e-3)
    y2 = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), "q4_k", k,
                        residual=torch.from_numpy(r).cuda())
    assert torch.equal(y, y2)  # the split-K sum runs in rank order: identical bits on every launch
    assert kernels.device_status() == 0


@pytest.mark.parametrize("n,k,mode", [(4096, 4096, "residual"), (2048, 4096, "swiglu"), (4096, 12288, "plain"),
                                      (6144, 4096, "qkv"), (4000, 4096, "plain"),
                                      # rank-local shapes of tensor parallelism over 4 / 8 GPUs: row-parallel
                                      # o_proj / down_proj with K = 1024 / 512 and 3072 / 1536, column-parallel
                                      # gate / up with 3072 / 1536 rows, QKV of 8 + 2 + 2 / 4 + 1 + 1 heads
                                      (4096, 512, "residual"), (4096, 1536, "residual"), (4096, 1024, "residual"),
                                      (1536, 4096, "swiglu"), (768, 4096, "qkv")])
def test_m1_qwen3_8b_shapes(oracle, n, k, mode):
    """M = 1 at Qwen3-8B sizes (8 warps split K of a 16-row block; K = 12288: three segments per warp;
    a ragged last row block).  Bound as for every matvec: 2e-3 against the double-precision oracle."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(n + k)
    x = rng.standard_normal((1, k)).astype(np.float16)
    xg = torch.from_numpy(x).cuda()
    if mode == "swiglu":
        pg = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
        pu = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
        g = oracle.matvec(pg, "q4_k", x).astype(np.float64)
        u = oracle.matvec(pu, "q4_k", x).astype(np.float64)
        ref = g / (1.0 + np.exp(-g)) * u
        y = kernels.linear_swiglu(xg, torch.from_numpy(pg).cuda(), torch.from_numpy(pu).cuda(), "q4_k", k)
        _tol_check(y.float().cpu().numpy(), ref, rel=4e-3)
    elif mode == "qkv":
        specs = [n * 2 // 3, n // 6, n // 6]  # q / k / v rows (6144: 4096 / 1024 / 1024)
        packed = [oracle.quantize(_weights(rng, r, k, special=False), "q4_k") for r in specs]
        outs = kernels.linear_multi(xg, [(torch.from_numpy(p).cuda(), "q4_k") for p in packed], k)
        for out, p in zip(outs, packed):
            _tol_check(out.float().cpu().numpy(), oracle.matvec(p, "q4_k", x))
    else:
        packed = oracle.quantize(_weights(rng, n, k, special=False), "q4_k")
        res = rng.standard_normal((1, n)).astype(np.float16) if mode == "residual" else None
        ref = oracle.matvec(packed, "q4_k", x) + (res.astype(np.float32) if res is not None else 0.0)
        y = kernels.linear(xg, torch.from_numpy(packed).cuda(), "q4_k", k,
                           residual=torch.from_numpy(res).cuda() if res is not None else None)
        _tol_check(y.float().cpu().numpy(), ref)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("m", [16, 64, 300])
@pytest.mark.parametrize("nk,res", [((4096, 4096), False), ((1030, 12288), True), ((520, 7680), False)])
def test_linear_q8_0_tensor_core(oracle, m, nk, res):
    """Q8_0 on the tcgen05 GEMM (272-byte windows of eight 34-byte blocks, d * q rounded to fp16): more
    tokens, a ragged row count, the residual epilogue and K = 7680 (the ASR conv_out projection)."""
    from torch2vk_b200 import kernels

    n, k = nk
    rng = np.random.default_rng(n + k + m)
    packed = oracle.quantize(_weights(rng, n, k), "q8_0")
    x = rng.standard_normal((m, k)).astype(np.float16)
    ref = oracle.matvec(packed, "q8_0", x)
    r = rng.standard_normal((m, n)).astype(np.float16) if res else None
    if res:
        ref = ref + r.astype(np.float32)
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), "q8_0", k,
                       residual=torch.from_numpy(r).cuda() if res else None)
    _tol_check(y.float().cpu().numpy(), ref, rel=4e-3)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("m", [1, 2, 3, 4, 9])
def test_matvec_is_deterministic(oracle, m):
    """Split-K partial sums meet in a fixed order: repeated launches give identical bits (the decode step,
    and so the greedy tokens, do not depend on warp scheduling)."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(m)
    n, k = 4096, 12288
    packed = torch.from_numpy(oracle.quantize(_weights(rng, n, k), "q4_k")).cuda()
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float16)).cuda()
    first = kernels.linear(x, packed, "q4_k", k)
    for _ in range(20):
        assert torch.equal(kernels.linear(x, packed, "q4_k", k), first)

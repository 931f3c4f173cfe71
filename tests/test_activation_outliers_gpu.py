"""GPU parity of the decode matvecs on activations with outliers.

The reference's matvec shaders read the fp16 x and accumulate
x * (d*sc*q - dmin*m) in fp32 (src/models/quantized_qwen3/shaders/
linear_nobias_q4_k_matvec_f32.py:107-197, linear_nobias_q6_k_matvec_f32.py:116-193,
linear_nobias_q8_0_matvec_f32.py:84-119).  Every output here is held to a
per-output bound that one extra fp16 rounding of every x (and of the stored
y) would produce:

    |y - ref| <= 2^-11 * (sum_k |w[n,k] * x[k]| + |ref[n]|)

where ref is the oracle's double-precision matvec on the same fp16 x and
packed weights.  Unlike a bound relative to |ref| or rms(ref), it does not
grow when an outlier of x meets a small weight.  Activation cases:

  (a) one value of +-100..2000 in every 32-value sub-block, the others ~1e-2;
  (b) a few fixed "massive activation" channels (+-800..3000) in N(0, 1);
  (c) as (a), with the weight columns of the outlier channels scaled by 1e-4,
      so that the small activations carry the output.

With a fused RMSNorm prologue the reference first rounds the normalized x to
fp16 (rms_norm_mul_f16_f32.py:22-115); the oracle does the same, and the norm
weight carries a few large channels.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

U = 2.0 ** -11


def _activations(rng: np.random.Generator, case: str, m: int, k: int) -> tuple[np.ndarray, np.ndarray]:
    """x [m, k] (fp16) and the outlier channel mask [k] of one case."""
    mask = np.zeros(k, dtype=bool)
    if case in ("a", "c"):
        x = rng.standard_normal((m, k)) * 0.01
        idx = np.arange(0, k, 32) + rng.integers(0, 32, k // 32)
        mask[idx] = True
        x[:, idx] = rng.choice([-1.0, 1.0], (m, idx.size)) * rng.uniform(100.0, 2000.0, (m, idx.size))
    else:
        x = rng.standard_normal((m, k))
        idx = rng.choice(k, 6, replace=False)
        mask[idx] = True
        x[:, idx] = np.array([1500.0, -800.0, 2500.0, -3000.0, 950.0, -1200.0])
    return x.astype(np.float16), mask


def _weights(rng: np.random.Generator, n: int, k: int, case: str, mask: np.ndarray) -> np.ndarray:
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if case == "c":
        w[:, mask] *= 1e-4
    return w


def _check(got: np.ndarray, ref: np.ndarray, absdot: np.ndarray, what: str) -> None:
    got = got.astype(np.float64)
    err = np.abs(got - ref)
    bound = U * (absdot + np.abs(ref)) + 1e-30
    ratio = err / bound
    worst = np.unravel_index(np.argmax(ratio), ratio.shape)
    assert ratio.max() <= 1.0, (
        f"{what}: err {err[worst]:.3e} > bound {bound[worst]:.3e} at {worst} (ref {ref[worst]:.4e}, "
        f"ratio {ratio.max():.2f})")


def _ref(oracle, packed: np.ndarray, kind: str, k: int, x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    w = oracle.dequantize(packed, kind, k).astype(np.float64)
    xd = x.astype(np.float64)
    return xd @ w.T, np.abs(xd) @ np.abs(w).T


@pytest.mark.parametrize("case", ["a", "b", "c"])
@pytest.mark.parametrize("kind", ["q4_k", "q6_k", "q8_0"])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
def test_matvec_outliers(oracle, case, kind, m):
    from torch2vk_b200 import kernels

    n, k = 384, 4096
    rng = np.random.default_rng(hash((case, kind, m)) % 2**32)
    x, mask = _activations(rng, case, m, k)
    packed = oracle.quantize(_weights(rng, n, k, case, mask), kind)
    ref, absdot = _ref(oracle, packed, kind, k, x)
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), kind, k)
    _check(y.float().cpu().numpy(), ref, absdot, f"{kind} M={m} case {case}")


@pytest.mark.parametrize("case", ["a", "c"])
def test_matvec_outliers_long_k(oracle, case):
    """K = 12288 (the 8B down projection): M = 1 and the per-token passes at M = 3."""
    from torch2vk_b200 import kernels

    n, k = 256, 12288
    for m in (1, 3):
        rng = np.random.default_rng(100 + m + ord(case))
        x, mask = _activations(rng, case, m, k)
        packed = oracle.quantize(_weights(rng, n, k, case, mask), "q4_k")
        ref, absdot = _ref(oracle, packed, "q4_k", k, x)
        y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), "q4_k", k)
        _check(y.float().cpu().numpy(), ref, absdot, f"q4_k K={k} M={m} case {case}")


def _normed(x: np.ndarray, nw: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    xf = x.astype(np.float32)
    r = 1.0 / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True) + np.float32(eps))
    return (xf * r * nw).astype(np.float16)


def _norm_weight(rng: np.random.Generator, k: int, mask: np.ndarray) -> np.ndarray:
    nw = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    big = rng.choice(k, 4, replace=False)
    nw[big] = np.array([40.0, -25.0, 60.0, 33.0], dtype=np.float32)
    return nw


@pytest.mark.parametrize("case", ["a", "b", "c"])
@pytest.mark.parametrize("m", [1, 2, 4])
def test_fused_norm_qkv_outliers(oracle, case, m):
    """QKV with the fused RMSNorm prologue (Q4_K q/k, Q6_K v)."""
    from torch2vk_b200 import kernels

    k = 4096
    rng = np.random.default_rng(hash(("qkv", case, m)) % 2**32)
    x, mask = _activations(rng, case, m, k)
    nw = _norm_weight(rng, k, mask)
    specs = [(512, "q4_k"), (256, "q4_k"), (256, "q6_k")]
    packed = [oracle.quantize(_weights(rng, n, k, case, mask), kind) for n, kind in specs]
    outs = kernels.linear_multi(torch.from_numpy(x).cuda(),
                                [(torch.from_numpy(p).cuda(), kind) for p, (_, kind) in zip(packed, specs)], k,
                                norm_weight=torch.from_numpy(nw).cuda())
    xn = _normed(x, nw)
    for (n, kind), p, o in zip(specs, packed, outs):
        ref, absdot = _ref(oracle, p, kind, k, xn)
        _check(o.float().cpu().numpy(), ref, absdot, f"qkv {kind} M={m} case {case}")


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_fused_norm_swiglu_outliers(oracle, case):
    """gate/up + SwiGLU with the fused RMSNorm prologue, M = 1."""
    from torch2vk_b200 import kernels

    n, k = 512, 4096
    rng = np.random.default_rng(hash(("swiglu", case)) % 2**32)
    x, mask = _activations(rng, case, 1, k)
    nw = _norm_weight(rng, k, mask)
    pg = oracle.quantize(_weights(rng, n, k, case, mask), "q4_k")
    pu = oracle.quantize(_weights(rng, n, k, case, mask), "q4_k")
    y = kernels.linear_swiglu(torch.from_numpy(x).cuda(), torch.from_numpy(pg).cuda(), torch.from_numpy(pu).cuda(),
                              "q4_k", k, norm_weight=torch.from_numpy(nw).cuda())
    xn = _normed(x, nw)
    g, gabs = _ref(oracle, pg, "q4_k", k, xn)
    u, uabs = _ref(oracle, pu, "q4_k", k, xn)
    sig = 1.0 / (1.0 + np.exp(-g))
    ref = g * sig * u
    # first-order propagation of the per-input bounds through silu(g) * u
    dsilu = sig * (1.0 + g * (1.0 - sig))
    absdot = np.abs(dsilu * u) * (gabs + np.abs(g)) + np.abs(g * sig) * (uabs + np.abs(u))
    _check(y.float().cpu().numpy(), ref, absdot, f"swiglu case {case}")


@pytest.mark.parametrize("case", ["a", "b", "c"])
@pytest.mark.parametrize("kind", ["q6_k", "q4_k"])
def test_lm_head_argmax_outliers(oracle, case, kind):
    """Fused final RMSNorm + LM-head argmax: the chosen row is the oracle's best
    unless the best and the chosen scores differ by less than their bounds."""
    from torch2vk_b200 import kernels

    n, k = 4000, 4096
    rng = np.random.default_rng(hash(("lm", case, kind)) % 2**32)
    x, mask = _activations(rng, case, 1, k)
    nw = _norm_weight(rng, k, mask)
    packed = oracle.quantize(_weights(rng, n, k, case, mask), kind)
    ps, pt = kernels.lm_head_argmax(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), kind, k,
                                    norm_weight=torch.from_numpy(nw).cuda())
    scores, tokens = ps.cpu().numpy()[0], pt.cpu().numpy()[0].astype(np.int64)
    ref, absdot = _ref(oracle, packed, kind, k, _normed(x, nw))
    ref, absdot = ref[0], absdot[0]
    bound = U * (absdot + np.abs(ref))
    for g in range(scores.size):
        row = int(tokens[g])
        assert 4 * g <= row < min(4 * g + 4, n)
        assert abs(scores[g] - ref[row]) <= bound[row], f"group {g}: score {scores[g]} vs {ref[row]}"
        best = 4 * g + int(np.argmax(ref[4 * g:4 * g + 4]))
        assert ref[best] - ref[row] <= bound[best] + bound[row], f"group {g}: row {row} instead of {best}"


@pytest.mark.parametrize("case", ["a", "b", "c"])
@pytest.mark.parametrize("m", [5, 8, 16])
def test_batched_q4k_outliers(oracle, case, m):
    """5..16 tokens of Q4_K (the batched kernel: K split over a thread-block cluster, tokens as mma columns)."""
    from torch2vk_b200 import kernels

    n, k = 300, 4096
    rng = np.random.default_rng(hash(("bt", case, m)) % 2**32)
    x, mask = _activations(rng, case, m, k)
    packed = oracle.quantize(_weights(rng, n, k, case, mask), "q4_k")
    ref, absdot = _ref(oracle, packed, "q4_k", k, x)
    res = rng.standard_normal((m, n)).astype(np.float16)
    y = kernels.linear(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), "q4_k", k,
                       residual=torch.from_numpy(res).cuda())
    ref = ref + res.astype(np.float64)
    _check(y.float().cpu().numpy(), ref, absdot + np.abs(res), f"batched q4_k M={m} case {case}")


@pytest.mark.parametrize("m,k", [(8, 12288), (9, 1024), (16, 3072)])
def test_batched_fused_norm_swiglu_and_qkv(oracle, m, k):
    """Batched kernel with the fused RMSNorm (the sum of squares shared across the cluster): gate/up + SwiGLU
    and a fused three-weight QKV, at the K of the 8B down projection and of the 0.6B shapes."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(m * 7 + k)
    x, mask = _activations(rng, "b", m, k)
    nw = _norm_weight(rng, k, mask)
    xn = _normed(x, nw)
    n = 200
    pg = oracle.quantize(_weights(rng, n, k, "b", mask), "q4_k")
    pu = oracle.quantize(_weights(rng, n, k, "b", mask), "q4_k")
    y = kernels.linear_swiglu(torch.from_numpy(x).cuda(), torch.from_numpy(pg).cuda(), torch.from_numpy(pu).cuda(),
                              "q4_k", k, norm_weight=torch.from_numpy(nw).cuda())
    g, gabs = _ref(oracle, pg, "q4_k", k, xn)
    u, uabs = _ref(oracle, pu, "q4_k", k, xn)
    sig = 1.0 / (1.0 + np.exp(-g))
    dsilu = sig * (1.0 + g * (1.0 - sig))
    absdot = np.abs(dsilu * u) * (gabs + np.abs(g)) + np.abs(g * sig) * (uabs + np.abs(u))
    _check(y.float().cpu().numpy(), g * sig * u, absdot, f"batched swiglu M={m} K={k}")
    specs = [(96, "q4_k"), (40, "q4_k"), (72, "q4_k")]
    packed = [oracle.quantize(_weights(rng, nn, k, "b", mask), kind) for nn, kind in specs]
    outs = kernels.linear_multi(torch.from_numpy(x).cuda(), [(torch.from_numpy(pk).cuda(), kd) for pk, (_, kd) in
                                                               zip(packed, specs)], k,
                                norm_weight=torch.from_numpy(nw).cuda())
    for (nn, kd), pk, o in zip(specs, packed, outs):
        ref, absdot = _ref(oracle, pk, kd, k, xn)
        _check(o.float().cpu().numpy(), ref, absdot, f"batched qkv M={m} K={k} n={nn}")

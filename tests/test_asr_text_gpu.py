"""GPU parity of the optimized Qwen3-ASR text-decoder programs served through the op table:
fused pair / triple Q4_K linears, the prefill attention that writes the caches
(sdpa_causal_cache_write_f16), the decode attention that writes the caches
(sdpa_decode_cache_write_f16) and the unfused RMSNorm chain's elementwise steps.

References: the oracle's block matvec (linears, 4e-3 as every tensor-core GEMM),
fp64 numpy attention over the same fp16 inputs (4e-3 relative + 2e-3 of the
output scale), and exact or 1e-6-relative checks for the elementwise steps.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(cls, b, s=None, pc=None, name="v", source="cuda"):
    from torch2vk_b200.runtime import optable

    v = SimpleNamespace(name=name, source=source, contract=SimpleNamespace(class_name=cls))
    optable.OPS[cls](None, v, b, s or {}, pc or {})


def _close(got, want, rel, abs_):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want)
    bound = rel * np.abs(want) + abs_
    worst = np.argmax(err - bound)
    assert np.all(err <= bound), f"max err {err.flat[worst]} > {bound.flat[worst]}"


def _attn(q, k, v, causal_rows=None):
    """q [NH, T, D], k / v [NK, S, D] (fp64); row t sees keys 0..t when causal_rows."""
    NH, T, D = q.shape
    NK, S, _ = k.shape
    out = np.zeros((NH, T, D))
    for h in range(NH):
        kh = h * NK // NH
        sc = q[h] @ k[kh].T / np.sqrt(D)
        if causal_rows:
            sc = np.where(np.arange(S)[None, :] <= np.arange(T)[:, None], sc, -np.inf)
        sc -= sc.max(-1, keepdims=True)
        p = np.exp(sc)
        out[h] = (p / p.sum(-1, keepdims=True)) @ v[kh]
    return out


@pytest.mark.parametrize("nw", [2, 3])
def test_linear_pair_triple(oracle, nw):
    rng = np.random.default_rng(nw)
    K, M, Ns = 1024, 16, [512, 256, 256][:nw]
    packed = [oracle.quantize((rng.standard_normal((n, K)) * 0.02).astype(np.float32), "q4_k") for n in Ns]
    x = rng.standard_normal((1, M, K)).astype(np.float16)
    outs = [torch.empty(1, M, n, dtype=torch.float16, device="cuda") for n in Ns]
    b = {"x": torch.from_numpy(x).cuda()}
    for i in range(nw):
        b[f"weight{i}"] = torch.from_numpy(packed[i]).cuda()
        b[f"output{i}"] = outs[i]
    _call("LinearNobiasQ4KPairProgram" if nw == 2 else "LinearNobiasQ4KTripleProgram", b, {"K": K})
    for i in range(nw):
        want = oracle.matvec(packed[i], "q4_k", x.reshape(M, K))
        rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
        _close(outs[i].float().cpu().numpy().reshape(M, -1), want, 4e-3, 4e-3 * rms)


def test_sdpa_causal_cache_write():
    rng = np.random.default_rng(3)
    B, NH, NK, T, S, D = 1, 16, 8, 37, 64, 128
    q = rng.standard_normal((B, NH, T, D)).astype(np.float16)
    k = rng.standard_normal((B, NK, T, D)).astype(np.float16)
    v = rng.standard_normal((B, T, NK, D)).astype(np.float16)
    kc = rng.standard_normal((B, NK, S, D)).astype(np.float16)
    vc = rng.standard_normal((B, NK, S, D)).astype(np.float16)
    pos = np.arange(10, 10 + T, dtype=np.int64)
    t = {n: torch.from_numpy(a.copy()).cuda() for n, a in dict(q=q, k=k, v=v, k_cache=kc, v_cache=vc).items()}
    t["cache_position"] = torch.from_numpy(pos).cuda()
    t["output"] = torch.empty(B, NH, T, D, dtype=torch.float16, device="cuda")
    _call("OptimizedQwen3SdpaCausalCacheWriteProgram", t, dict(B=B, NH=NH, NK=NK, T=T, S=S, D=D))
    want_kc, want_vc = kc.copy(), vc.copy()
    want_kc[0][:, pos] = k[0]
    want_vc[0][:, pos] = v[0].transpose(1, 0, 2)
    assert np.array_equal(t["k_cache"].cpu().numpy(), want_kc)
    assert np.array_equal(t["v_cache"].cpu().numpy(), want_vc)
    want = _attn(q[0].astype(np.float64), k[0].astype(np.float64), v[0].transpose(1, 0, 2).astype(np.float64), True)
    _close(t["output"].float().cpu().numpy()[0], want, 4e-3, 2e-3 * float(np.abs(want).max()))


@pytest.mark.parametrize("pos", [20, 63])
def test_sdpa_decode_cache_write_f16(pos):
    rng = np.random.default_rng(pos)
    B, NH, NK, S, D = 1, 16, 8, 64, 128
    q = rng.standard_normal((B, NH, 1, D)).astype(np.float16)
    nk = rng.standard_normal((B, NK, 1, D)).astype(np.float16)
    nv = rng.standard_normal((B, 1, NK, D)).astype(np.float16)
    kc = rng.standard_normal((B, NK, S, D)).astype(np.float16)
    vc = rng.standard_normal((B, NK, S, D)).astype(np.float16)
    t = {n: torch.from_numpy(a.copy()).cuda() for n, a in dict(q=q, new_k=nk, new_v=nv, k_cache=kc, v_cache=vc).items()}
    t["output"] = torch.empty(B, NH, 1, D, dtype=torch.float16, device="cuda")
    _call("SdpaDecodeCacheWriteF16Program", t, dict(B=B, NH=NH, NK=NK, S=S, D=D, T=1), {"cache_position": pos})
    kc[0][:, pos] = nk[0][:, 0]
    vc[0][:, pos] = nv[0][0]
    assert np.array_equal(t["k_cache"].cpu().numpy(), kc) and np.array_equal(t["v_cache"].cpu().numpy(), vc)
    want = _attn(q[0].astype(np.float64), kc[0][:, :pos + 1].astype(np.float64), vc[0][:, :pos + 1].astype(np.float64))
    _close(t["output"].float().cpu().numpy()[0], want, 4e-3, 2e-3 * float(np.abs(want).max()))


def test_unfused_rms_norm_chain():
    """pow -> mean -> add eps -> rsqrt -> mul by row -> mul by weight, as the exported text norm runs it."""
    rng = np.random.default_rng(8)
    T, H = 7, 1024
    x = (rng.standard_normal((1, T, H)) * 3).astype(np.float16)
    w = (rng.random(H) + 0.5).astype(np.float32)
    tx, tw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    sq = torch.empty(1, T, H, device="cuda")
    _call("ExportPowScalarF32Program", {"x": tx, "output": sq})
    x32 = x.astype(np.float32)
    assert np.array_equal(sq.cpu().numpy(), x32 * x32)
    mean = torch.empty(1, T, 1, device="cuda")
    _call("ExportMeanDimProgram", {"x": sq, "output": mean})
    _close(mean.cpu().numpy(), (x32.astype(np.float64) ** 2).mean(-1, keepdims=True), 1e-5, 0)
    eps = torch.empty_like(mean)
    _call("ExportAddScalarProgram", {"x": mean, "output": eps}, pc={"scalar": 1e-6, "N": T})
    assert np.array_equal(eps.cpu().numpy(), mean.cpu().numpy() + np.float32(1e-6))
    r = torch.empty_like(mean)
    _call("ExportRsqrtF32Program", {"x": eps, "output": r})
    _close(r.cpu().numpy(), 1 / np.sqrt(eps.cpu().numpy().astype(np.float64)), 1e-6, 0)
    normed = torch.empty(1, T, H, dtype=torch.float16, device="cuda")
    _call("ExportMulBroadcastLastProgram", {"x": tx, "y": r, "output": normed}, pc={"H": H, "N": T * H})
    assert np.array_equal(normed.cpu().numpy(), (x32 * r.cpu().numpy()).astype(np.float16))
    out = torch.empty_like(normed)
    _call("ExportMulLeftBroadcastF32XProgram", {"x": tw, "y": normed, "output": out}, pc={"H": H, "N": T * H})
    assert np.array_equal(out.cpu().numpy(), (normed.cpu().numpy().astype(np.float32) * w).astype(np.float16))

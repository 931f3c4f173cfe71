"""GPU parity of the optimized Qwen3 fp32-activation prefill programs (llama.cpp-style chain).

Checked against oracle/prefill32_ref.py (CPU restatements of the reference
shaders) and the oracle's block matvec.  Bounds, per test:
* integer / copy work (mask classifier, cache writes, casts, slices): exact;
* fp32 elementwise and norms: 1e-5 relative (rsqrt / exp approximations);
* the fp32 GEMM: x is rounded to fp16 (as the reference's cooperative-matrix
  operands are) and multiplied on the tensor cores, 4e-3 as every tensor-core GEMM;
* attention: fp16 K / V and fp16-rounded q, probabilities split into fp16 high +
  low parts: 4e-3 relative + 2e-3 absolute of the output scale.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import prefill32_ref as ref

pytestmark = pytest.mark.gpu


def _close(got, want, rel, abs_=0.0):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bound = rel * np.abs(want) + abs_
    worst = np.argmax(err - bound)
    assert np.all(err <= bound), f"max err {err.flat[worst]} > bound {bound.flat[worst]} (want {want.flat[worst]})"


def _weights(rng, n, k):
    return (rng.standard_normal((n, k)) * 0.02).astype(np.float32)


@pytest.mark.parametrize("kind", ["q4_k", "q6_k"])
@pytest.mark.parametrize("m", [3, 16, 130])
@pytest.mark.parametrize("nk", [(1030, 2048), (256, 4096)])
def test_linear_f32(oracle, kind, m, nk):
    """LlamaMatmulQ{4,6}KF32Program: fp32 x -> fp32 y."""
    from torch2vk_b200 import kernels

    n, k = nk
    rng = np.random.default_rng(n + k + m)
    packed = oracle.quantize(_weights(rng, n, k), kind)
    x = rng.standard_normal((1, m, k)).astype(np.float32)
    want = oracle.matvec(packed, kind, x.reshape(m, k).astype(np.float16))
    y = kernels.linear_f32(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), kind, k)
    assert y.dtype == torch.float32 and tuple(y.shape) == (1, m, n)
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    _close(y.cpu().numpy().reshape(m, n), want, 4e-3, 4e-3 * rms)


@pytest.mark.parametrize("rows,h", [(37, 1024), (5, 4096), (3, 1027)])
def test_rms_norm_f32(rows, h):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(rows * h)
    x = (rng.standard_normal((1, rows, h)) * 3).astype(np.float32)
    w = (rng.random(h) + 0.5).astype(np.float32)
    y = kernels.rms_norm_f32(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), 1e-6)
    _close(y.cpu().numpy(), ref.rms_norm_mul(x, w), 1e-5, 1e-6)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("d", [128, 64])
def test_rms_norm_rope_token_f32(out_dtype, d):
    """OptimizedQwen3RmsNormRopeTokenF32Program / ...F32ToF16Program."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(d)
    B, T, G = 2, 37, 8
    x = (rng.standard_normal((B, T, G, d)) * 2).astype(np.float32)
    w = (rng.random(d) + 0.5).astype(np.float32)
    ang = rng.random((B, T, d)).astype(np.float32) * 6
    cos, sin = np.cos(ang).astype(np.float16), np.sin(ang).astype(np.float16)
    out = torch.empty(B, T, G, d, dtype=out_dtype, device="cuda")
    kernels.rms_norm_rope_f32(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(cos).cuda(),
                              torch.from_numpy(sin).cuda(), out)
    want = ref.rms_norm_rope_token(x, w, cos, sin)
    if out_dtype == torch.float32:
        _close(out.cpu().numpy(), want, 1e-5, 1e-5)
    else:
        _close(out.float().cpu().numpy(), want, 1e-3, 1e-3)


@pytest.mark.parametrize("n", [4096 * 3, 4099])
def test_add_swiglu_f32(n):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(n)
    a = (rng.standard_normal(n) * 4).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    assert np.array_equal(kernels.add_f32(ta, tb).cpu().numpy(), a + b)
    a64 = a.astype(np.float64)
    _close(kernels.swiglu_f32(ta, tb).cpu().numpy(), a64 / (1 + np.exp(-a64)) * b, 1e-5, 1e-7)


def test_cast_and_slice_last():
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(1)
    x = (rng.standard_normal((3, 17, 260)) * 100).astype(np.float32)
    tx = torch.from_numpy(x).cuda()
    h = torch.empty(3, 17, 260, dtype=torch.float16, device="cuda")
    kernels.cast(tx, h)
    assert np.array_equal(h.cpu().numpy(), x.astype(np.float16))
    back = torch.empty_like(tx)
    kernels.cast(h, back)
    assert np.array_equal(back.cpu().numpy(), x.astype(np.float16).astype(np.float32))
    last = torch.empty(3, 1, 260, dtype=torch.float16, device="cuda")
    kernels.slice_last_f32_to_f16(tx, last)
    assert np.array_equal(last.cpu().numpy(), x[:, -1:, :].astype(np.float16))


@pytest.mark.parametrize("ncaches", [2, 3])
def test_value_cache_write_f32(ncaches):
    """Positions past a cache's extent are skipped for that cache only (as the reference)."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(ncaches)
    B, T, H, D = 1, 9, 8, 128
    lens = [64, 40, 16][:ncaches]
    src = rng.standard_normal((B, T, H, D)).astype(np.float32)
    pos = np.array([3, 0, 15, 16, 39, 40, 63, 20, 7], np.int64)
    caches = [(rng.standard_normal((B, s, H, D))).astype(np.float16) for s in lens]
    dev = [torch.from_numpy(c.copy()).cuda() for c in caches]
    kernels.value_cache_write_f32(torch.from_numpy(src).cuda(), torch.from_numpy(pos).cuda(), dev)
    ref.value_cache_write(caches, src, pos)
    for got, want in zip(dev, caches):
        assert np.array_equal(got.cpu().numpy(), want)


def _masks():
    rng = np.random.default_rng(5)
    yield "causal_full", ref.causal_mask(0, 100, 100)
    yield "causal_tail", ref.causal_mask(512, 9, 576)
    yield "wide", ref.causal_mask(700, 300, 1100)
    m = np.zeros((40, 2100), np.float16)
    m[:, 64:128] = -np.inf                            # one all-masked column block
    m[16:32, 256:320] = np.float16(-60000.0)          # finite, not "masked"
    m[:, 1000:1005] = rng.standard_normal((40, 5)).astype(np.float16)
    m[5, 2000] = -np.inf
    yield "mixed", m


@pytest.mark.parametrize("name,mask", list(_masks()), ids=[n for n, _ in _masks()])
def test_fa_mask_opt(name, mask):
    from torch2vk_b200 import kernels

    T, S = mask.shape
    want = ref.fa_mask_opt(mask)
    out = torch.full(want.shape, -1, dtype=torch.int32, device="cuda")
    kernels.fa_mask_opt(torch.from_numpy(mask).cuda(), out)
    got = out.cpu().numpy().view(np.uint32)
    assert np.array_equal(got, want), f"{name}: {np.argwhere(got != want)[:4].tolist()}"


@pytest.mark.parametrize("case", ["tail", "chunk", "mixed_mask", "gqa1"])
def test_attn_prefill_masked_f32(case):
    """LlamaFlashAttnF32F16F16Program, with and without the classifier's codes (same result)."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(len(case))
    NH, NK, D = (8, 8, 128) if case == "gqa1" else (32, 8, 128)
    if case == "tail":
        B, T, S, mask = 1, 9, 576, ref.causal_mask(512, 9, 576)
    elif case == "chunk":
        B, T, S, mask = 1, 200, 256, ref.causal_mask(0, 200, 256)
    elif case == "gqa1":
        B, T, S, mask = 2, 70, 192, ref.causal_mask(100, 70, 192)
    else:
        B, T, S = 1, 40, 300
        mask = (rng.standard_normal((T, S)) * 2).astype(np.float16)
        mask[:, 64:192] = -np.inf
        mask[:, 0] = 0
    q = rng.standard_normal((B, T, NH, D)).astype(np.float32)
    k = rng.standard_normal((B, S, NK, D)).astype(np.float16)
    v = rng.standard_normal((B, S, NK, D)).astype(np.float16)
    scale = 1.0 / np.sqrt(D)
    want = ref.flash_attn(q.astype(np.float16).astype(np.float32), k, v, mask, scale)
    tq, tk, tv, tm = (torch.from_numpy(a).cuda() for a in (q, k, v, mask))
    opt = torch.zeros((T + 15) // 16, (S + 1023) // 1024, dtype=torch.int32, device="cuda")
    kernels.fa_mask_opt(tm, opt)
    scale_out = float(np.abs(want).max())
    for mo in (None, opt):
        out = torch.full((B, T, NH, D), float("nan"), device="cuda")
        kernels.attn_prefill_masked_f32(tq, tk, tv, tm, mo, out, scale=scale)
        _close(out.cpu().numpy(), want, 4e-3, 2e-3 * scale_out)


def test_embedding_f32(oracle):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(11)
    vocab, h = 300, 1024
    packed = oracle.quantize(_weights(rng, vocab, h), "q4_k")
    table = oracle.dequantize(packed, "q4_k", h)
    ids = np.array([[0, 299, 17, 17, 150]], np.int64)
    out = kernels.embedding_f32(torch.from_numpy(packed).cuda(), "q4_k", torch.from_numpy(ids).cuda(), h, vocab)
    _close(out.cpu().numpy(), table[ids], 1e-6, 1e-9)


def test_prefill32_ops_through_optable(oracle):
    """The op-table entries (the drop-in glue) on real buffers: field names, symbols, push constants."""
    from torch2vk_b200.runtime import optable

    rng = np.random.default_rng(2)

    def call(cls, b, s=None, pc=None, name="v"):
        v = SimpleNamespace(name=name, contract=SimpleNamespace(class_name=cls))
        optable.OPS[cls](None, v, b, s or {}, pc or {})

    T, H, N = 12, 1024, 512
    packed = oracle.quantize(_weights(rng, N, H), "q4_k")
    x = rng.standard_normal((1, T, H)).astype(np.float32)
    y = torch.empty(1, T, N, device="cuda")
    call("LlamaMatmulQ4KF32Program", {"x": torch.from_numpy(x).cuda(), "weight": torch.from_numpy(packed).cuda(),
                                      "output": y}, {"K": H, "N": N})
    want = oracle.matvec(packed, "q4_k", x.reshape(T, H).astype(np.float16))
    _close(y.cpu().numpy().reshape(T, N), want, 4e-3, 4e-3 * float(np.sqrt(np.mean(want ** 2))))

    w = (rng.random(H) + 0.5).astype(np.float32)
    o = torch.empty(1, T, H, device="cuda")
    call("OptimizedQwen3RmsNormMulF32Program", {"x": torch.from_numpy(x).cuda(), "weight": torch.from_numpy(w).cuda(),
                                                "output": o})
    _close(o.cpu().numpy(), ref.rms_norm_mul(x, w), 1e-5, 1e-6)

    a = torch.from_numpy(x).cuda()
    o2 = torch.empty_like(a)
    call("AddF32PrefillProgram", {"x": a, "y": o, "output": o2})
    assert torch.equal(o2, a + o)
    call("SwigluF32Program", {"gate": a, "up": o, "output": o2})
    _close(o2.cpu().numpy(), (x / (1 + np.exp(-x.astype(np.float64)))) * o.cpu().numpy(), 1e-5, 1e-7)

    mask = ref.causal_mask(4, T, 64)
    W, R = 1, 1
    mo = torch.full((W, R), -1, dtype=torch.int32, device="cuda")
    call("OptimizedQwen3FaMaskOptF16Program", {"mask": torch.from_numpy(mask).cuda(), "output": mo},
         {"W": W, "R": R, "S": 64, "T": T})
    assert np.array_equal(mo.cpu().numpy().view(np.uint32).reshape(R, W), ref.fa_mask_opt(mask))

    q = rng.standard_normal((1, T, 16, 128)).astype(np.float32)
    kc = rng.standard_normal((1, 64, 8, 128)).astype(np.float16)
    vc = rng.standard_normal((1, 64, 8, 128)).astype(np.float16)
    out = torch.empty(1, T, 16, 128, device="cuda")
    call("LlamaFlashAttnF32F16F16Program",
         {"q": torch.from_numpy(q).cuda(), "k": torch.from_numpy(kc).cuda(), "v": torch.from_numpy(vc).cuda(),
          "mask": torch.from_numpy(mask).cuda(), "sink": torch.from_numpy(q).cuda(), "output": out, "mask_opt": mo},
         {}, {"scale": 1 / np.sqrt(128), "mask_n_head_log2": 16, "logit_softcap": 0.0, "max_bias": 0.0})
    want = ref.flash_attn(q.astype(np.float16).astype(np.float32), kc, vc, mask, 1 / np.sqrt(128))
    _close(out.cpu().numpy(), want, 4e-3, 2e-3 * float(np.abs(want).max()))

    src = rng.standard_normal((1, T, 8, 128)).astype(np.float32)
    ca, cb = torch.zeros(1, 64, 8, 128, dtype=torch.float16, device="cuda"), torch.zeros(
        1, 8, 8, 128, dtype=torch.float16, device="cuda")
    pos = np.arange(4, 4 + T, dtype=np.int64)
    call("OptimizedQwen3TokenMajorValueCacheWriteF32ToF16PairProgram",
         {"cache_a": ca, "cache_b": cb, "cache_position": torch.from_numpy(pos).cuda(), "src": torch.from_numpy(src).cuda()})
    na, nb = np.zeros((1, 64, 8, 128), np.float16), np.zeros((1, 8, 8, 128), np.float16)
    ref.value_cache_write([na, nb], src, pos)
    assert np.array_equal(ca.cpu().numpy(), na) and np.array_equal(cb.cpu().numpy(), nb)

"""GPU parity of the decode-path kernels against plain PyTorch fp32 references.

Tolerances are written per test: fp16 storage of results bounds every
comparison at a few fp16 ulps of the reference magnitude.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(got: torch.Tensor, ref: torch.Tensor, rel: float = 4e-3, abs_: float = 2e-3) -> None:
    got = got.float().cpu()
    ref = ref.float().cpu()
    err = (got - ref).abs()
    bound = rel * ref.abs() + abs_
    bad = err > bound
    assert not bool(bad.any()), f"max err {float(err.max())} (bound at worst {float(bound.flatten()[err.argmax()])})"


@pytest.mark.parametrize("rows,cols", [(37, 1024), (1, 4096), (32, 4096), (5, 12288), (3, 1028)])
def test_rms_norm(rows, cols):
    """One CTA per row for rows of up to 8192 values (multiples of 8), one warp per row otherwise."""
    from torch2vk_b200 import kernels

    torch.manual_seed(0)
    x = torch.randn(rows, cols, device="cuda", dtype=torch.float16) * 3
    w = torch.rand(cols, device="cuda") + 0.5
    y = kernels.rms_norm(x, w, 1e-6)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    _close(y, ref)


def _rope_ref(x: torch.Tensor, w: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor, eps: float) -> torch.Tensor:
    # x [M, H, D] fp32; pos [M]
    xn = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w
    ang = pos.float()[:, None] * inv_freq[None, :]
    emb = torch.cat([ang, ang], dim=-1)
    cos, sin = emb.cos()[:, None, :], emb.sin()[:, None, :]
    half = x.shape[-1] // 2
    rot = torch.cat([-xn[..., half:], xn[..., :half]], dim=-1)
    return xn * cos + rot * sin


@pytest.mark.parametrize("layout", ["token_major", "head_major"])
def test_qk_norm_rope_cache(layout):
    from torch2vk_b200 import kernels
    from torch2vk_b200.qwen3 import Qwen3Config, inv_freq

    torch.manual_seed(1)
    B, T, NH, NK, D, S = 2, 5, 16, 8, 128, 64
    cfg = Qwen3Config(hidden=1024, layers=1, heads=NH, kv_heads=NK, head_dim=D, intermediate=3072, vocab=16)
    freqs = inv_freq(cfg)
    q = torch.randn(B * T, NH * D, device="cuda", dtype=torch.float16)
    k = torch.randn(B * T, NK * D, device="cuda", dtype=torch.float16)
    v = torch.randn(B * T, NK * D, device="cuda", dtype=torch.float16)
    qw = torch.rand(D, device="cuda") + 0.5
    kw = torch.rand(D, device="cuda") + 0.5
    shape = (B, S, NK, D) if layout == "token_major" else (B, NK, S, D)
    kc = torch.zeros(shape, device="cuda", dtype=torch.float16)
    vc = torch.zeros(shape, device="cuda", dtype=torch.float16)
    positions = torch.tensor([3, 40], device="cuda", dtype=torch.int32)
    qo = kernels.qk_norm_rope_cache(q, k, v, qw, kw, kc, vc, positions, freqs.cuda(), batch=B, tokens=T, n_heads=NH,
                                    n_kv=NK, head_dim=D, layout=layout)
    pos = (positions.cpu()[:, None] + torch.arange(T)[None, :]).reshape(-1)
    ref_q = _rope_ref(q.float().cpu().view(B * T, NH, D), qw.cpu(), pos, freqs, 1e-6)
    ref_k = _rope_ref(k.float().cpu().view(B * T, NK, D), kw.cpu(), pos, freqs, 1e-6)
    _close(qo.view(B * T, NH, D), ref_q)
    kc_t = kc if layout == "token_major" else kc.transpose(1, 2)
    vc_t = vc if layout == "token_major" else vc.transpose(1, 2)
    for b in range(B):
        for t in range(T):
            p = int(positions[b]) + t
            _close(kc_t[b, p], ref_k[b * T + t])
            _close(vc_t[b, p], v.float().cpu().view(B * T, NK, D)[b * T + t], rel=0, abs_=0)


def _attn_ref(q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, lens: list[int], NH: int, NK: int) -> torch.Tensor:
    # q [B, NH, D]; caches [B, S, NK, D]
    B, _, D = q.shape
    out = torch.empty(B, NH, D)
    g = NH // NK
    for b in range(B):
        kk = kc[b, : lens[b]].float().cpu()  # [L, NK, D]
        vv = vc[b, : lens[b]].float().cpu()
        for h in range(NH):
            s = (kk[:, h // g, :] @ q[b, h].float().cpu()) / math.sqrt(D)
            p = torch.softmax(s, dim=0)
            out[b, h] = p @ vv[:, h // g, :]
    return out


@pytest.mark.parametrize("NH,NK", [(16, 8), (32, 8)])
@pytest.mark.parametrize("splits", [1, 4, 16])
def test_attn_decode(NH, NK, splits):
    from torch2vk_b200 import kernels

    torch.manual_seed(2)
    B, D, S = 3, 128, 700
    q = torch.randn(B, NH * D, device="cuda", dtype=torch.float16)
    kc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    vc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    positions = torch.tensor([0, 255, 699], device="cuda", dtype=torch.int32)
    out = kernels.attn_decode(q, kc, vc, positions, batch=B, n_heads=NH, n_kv=NK, head_dim=D, max_len=S,
                              splits=splits)
    ref = _attn_ref(q.view(B, NH, D), kc, vc, [1, 256, 700], NH, NK)
    _close(out.view(B, NH, D), ref)


@pytest.mark.parametrize("B,T,NH,NK,S,base", [(2, 37, 16, 8, 96, [0, 20]), (2, 150, 32, 8, 900, [0, 700]),
                                                (1, 129, 64, 8, 200, [64])])
def test_attn_prefill(B, T, NH, NK, S, base):
    """Causal GQA prefill (64-query tiles on tensor cores, ragged last tile, cache prefix) vs an fp32 reference."""
    from torch2vk_b200 import kernels

    torch.manual_seed(3)
    D = 128
    q = torch.randn(B * T, NH * D, device="cuda", dtype=torch.float16)
    kc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    vc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    positions = torch.tensor(base, device="cuda", dtype=torch.int32)
    out = kernels.attn_prefill(q, kc, vc, positions, batch=B, tokens=T, n_heads=NH, n_kv=NK, head_dim=D)
    qq = q.view(B, T, NH, D)
    ref = torch.empty(B, T, NH, D)
    for b in range(B):
        for t in range(T):
            ref[b, t] = _attn_ref(qq[b, t][None], kc[b:b + 1], vc[b:b + 1], [base[b] + t + 1], NH, NK)[0]
    _close(out.view(B, T, NH, D), ref)


@pytest.mark.parametrize("T", [2048, 8192])
def test_attn_prefill_long(T):
    """Causal GQA prefill at the attention sweep's long prompts (2k / 8k, batch 1, 32 Q / 8 KV heads) vs a
    plain PyTorch fp32 reference computed on the GPU."""
    from torch2vk_b200 import kernels

    torch.manual_seed(T)
    B, NH, NK, D = 1, 32, 8, 128
    q = torch.randn(B * T, NH * D, device="cuda", dtype=torch.float16)
    kc = torch.randn(B, T, NK, D, device="cuda", dtype=torch.float16)
    vc = torch.randn(B, T, NK, D, device="cuda", dtype=torch.float16)
    positions = torch.zeros(B, device="cuda", dtype=torch.int32)
    out = kernels.attn_prefill(q, kc, vc, positions, batch=B, tokens=T, n_heads=NH, n_kv=NK, head_dim=D)
    qq = q.view(T, NH, D).float().transpose(0, 1)                      # [NH, T, D]
    kk = kc[0].float().transpose(0, 1).repeat_interleave(NH // NK, 0)  # [NH, T, D]
    vv = vc[0].float().transpose(0, 1).repeat_interleave(NH // NK, 0)
    causal = torch.full((T, T), float("-inf"), device="cuda").triu(1)
    ref = torch.empty(NH, T, D, device="cuda")
    for h in range(NH):
        p = torch.softmax(qq[h] @ kk[h].T / math.sqrt(D) + causal, dim=-1)
        ref[h] = p @ vv[h]
    _close(out.view(T, NH, D), ref.transpose(0, 1))


def test_embedding_f16_and_q4k(oracle):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(4)
    V, H = 300, 512
    w = (rng.standard_normal((V, H)) * 0.02).astype(np.float32)
    ids = torch.tensor([0, 299, 17, 17, 150], dtype=torch.int64, device="cuda")
    emb16 = torch.from_numpy(w.astype(np.float16)).cuda()
    out = kernels.embedding(emb16, "f16", ids, H, V)
    assert torch.equal(out.cpu(), emb16.cpu()[ids.cpu()])
    packed = oracle.quantize(w, "q4_k")
    out = kernels.embedding(torch.from_numpy(packed).cuda(), "q4_k", ids, H, V)
    want = oracle.dequantize(packed, "q4_k", H)[ids.cpu().numpy()].astype(np.float16)
    assert np.array_equal(out.cpu().numpy(), want)


# (q6_k, 512) and (q8_0, 1088) have rows whose byte length is not a multiple of
# 16, so they take the direct (non-bulk-copy) kernel; N = 4099 leaves a ragged group.
@pytest.mark.parametrize("kind,K,N", [("q6_k", 1024, 4112), ("q6_k", 4096, 4112), ("q4_k", 1024, 4112),
                                      ("q6_k", 512, 4099), ("q8_0", 1088, 4099)])
@pytest.mark.parametrize("M", [2, 3, 4])
def test_lm_head_argmax_and_select(oracle, kind, K, N, M):
    """2..4 tokens in one pass of the weights (Q6_K / Q8_0: qmv_x16_kernel<2 or 4>)."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(5)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[777] = w[123]          # an exact duplicate row: tie -> lower id
    packed = oracle.quantize(w, kind)
    x = rng.standard_normal((M, K)).astype(np.float16)
    x[1] = x[0]
    logits = oracle.matvec(packed, kind, x)
    xg = torch.from_numpy(x).cuda()
    ps, pt = kernels.lm_head_argmax(xg, torch.from_numpy(packed).cuda(), kind, K)
    assert ps.shape == (M, (N + 3) // 4)
    ps_c, pt_c = ps.cpu().numpy(), pt.cpu().numpy()
    for m in range(M):
        for g in range(ps_c.shape[1]):
            rows = logits[m, 4 * g:4 * g + 4]
            assert pt_c[m, g] == 4 * g + int(np.argmax(rows)) or abs(float(rows.max()) - float(ps_c[m, g])) < 1e-3
        assert abs(float(ps_c[m].max()) - float(logits[m].max())) <= 2e-3 * (abs(float(logits[m].max())) + 1)
    eos = torch.tensor([int(pt_c[0, np.argmax(ps_c[0])]), 5], dtype=torch.int64, device="cuda")
    nxt, done = kernels.token_select(ps, pt, eos)
    assert int(nxt[0]) == int(np.argmax(logits[0])) or logits[0].max() - np.sort(logits[0])[-2] < 1e-3
    assert int(nxt[0]) == int(nxt[1]) and int(done[0]) == 1 and int(done[1]) == 1


@pytest.mark.parametrize("kind,K,N,M", [("q6_k", 4096, 4099, 8), ("q6_k", 4096, 8192, 32), ("q4_k", 4096, 4099, 20),
                                        ("q6_k", 2048, 1000, 5), ("q6_k", 1024, 8192, 9), ("q6_k", 2560, 1000, 40)])
def test_lm_head_argmax_tensor_core(oracle, kind, K, N, M):
    """M > 4: the LM head runs on the tcgen05 GEMM (fp16 operands) with the argmax epilogue.

    Scores are fp16-operand dot products: each partial may differ from the double-precision oracle by
    4e-3 relative (the tensor-core GEMM bound), and a group's reported row must be the oracle's argmax
    unless the two best rows of the group are that close."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(6)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[777 % N] = w[123]
    packed = oracle.quantize(w, kind)
    x = rng.standard_normal((M, K)).astype(np.float16)
    nw = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    xf = x.astype(np.float64)
    xn = (xf / np.sqrt(np.mean(xf * xf, axis=1, keepdims=True) + 1e-6) * nw).astype(np.float16)
    logits = oracle.matvec(packed, kind, xn)
    ps, pt = kernels.lm_head_argmax(torch.from_numpy(x).cuda(), torch.from_numpy(packed).cuda(), kind, K,
                                    norm_weight=torch.from_numpy(nw).cuda())
    ps_c, pt_c = ps.cpu().numpy(), pt.cpu().numpy()
    scale = float(np.sqrt(np.mean(logits.astype(np.float64) ** 2)))
    for m in range(M):
        for g in range(ps_c.shape[1]):
            rows = logits[m, 4 * g:4 * g + 4]
            tol = 4e-3 * (abs(float(rows.max())) + scale)
            assert abs(float(ps_c[m, g]) - float(rows.max())) <= tol
            best = int(np.argmax(rows))
            assert pt_c[m, g] == 4 * g + best or float(rows.max()) - float(rows[pt_c[m, g] - 4 * g]) <= 2 * tol
    assert kernels.device_status() == 0


def test_token_select_tie_breaks_to_lower_id():
    from torch2vk_b200 import kernels

    G = 5000
    ps = torch.full((1, G), -1.0, device="cuda")
    pt = torch.arange(G, dtype=torch.int32, device="cuda")[None].contiguous()
    ps[0, 4321] = 3.0
    ps[0, 1234] = 3.0
    nxt, done = kernels.token_select(ps, pt, torch.tensor([-1], dtype=torch.int64, device="cuda"))
    assert int(nxt[0]) == 1234 and int(done[0]) == 0


def test_token_store_and_advance():
    from torch2vk_b200 import kernels

    B, G = 2, 4
    gen = torch.zeros(B, G, dtype=torch.int64, device="cuda")
    length = torch.zeros(B, dtype=torch.int32, device="cuda")
    stopped = torch.zeros(B, dtype=torch.int32, device="cuda")
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.tensor([7, 9], dtype=torch.int32, device="cuda")
    seq = [([11, 21], [0, 0]), ([12, 22], [1, 0]), ([13, 23], [0, 0]), ([14, 24], [0, 0]), ([15, 25], [0, 0])]
    for toks, dn in seq:
        kernels.token_store(torch.tensor(toks, device="cuda"), torch.tensor(dn, dtype=torch.int32, device="cuda"),
                            gen, length, stopped, token_index_dev=idx, stop_on_eos=True)
        kernels.advance_positions(pos, idx)
    assert gen.cpu().tolist() == [[11, 12, 0, 0], [21, 22, 23, 24]]
    assert length.cpu().tolist() == [2, 4] and stopped.cpu().tolist() == [1, 0]
    assert pos.cpu().tolist() == [12, 14] and int(idx[0]) == 5


def test_elementwise_add_swiglu():
    from torch2vk_b200 import kernels

    torch.manual_seed(6)
    a = torch.randn(1027, device="cuda", dtype=torch.float16)
    b = torch.randn(1027, device="cuda", dtype=torch.float16)
    _close(kernels.add(a, b), a.float() + b.float())
    silu = (a.float() / (1 + torch.exp(-a.float()))).half().float()
    _close(kernels.swiglu(a, b), silu * b.float())


@pytest.mark.parametrize("layout", ["token_major", "head_major"])
@pytest.mark.parametrize("NH,NK,splits", [(32, 8, 1), (32, 8, 5), (32, 8, 8), (32, 8, 23), (16, 8, 7), (8, 8, 3),
                                          (64, 8, 8), (64, 8, 9), (4, 1, 8), (8, 2, 8)])
def test_attn_decode_fused_matches_unfused_chain(NH, NK, splits, layout):
    """One-launch decode attention == qk_norm_rope_cache + attn_decode (same caches after, outputs close).

    splits <= 8: one thread-block cluster per (sequence, KV head), combined through distributed shared
    memory; more splits: partials in a global workspace, combined by the last arriving warp."""
    from torch2vk_b200 import kernels
    from torch2vk_b200.qwen3 import Qwen3Config, inv_freq

    torch.manual_seed(7)
    B, D, S = 3, 128, 700
    cfg = Qwen3Config.qwen3_0_6b()
    inv = inv_freq(cfg).cuda()
    q = torch.randn(B, NH * D, device="cuda", dtype=torch.float16)
    k = torch.randn(B, NK * D, device="cuda", dtype=torch.float16)
    v = torch.randn(B, NK * D, device="cuda", dtype=torch.float16)
    qw = 1 + 0.1 * torch.randn(D, device="cuda")
    kw = 1 + 0.1 * torch.randn(D, device="cuda")
    shape = (B, S, NK, D) if layout == "token_major" else (B, NK, S, D)
    kc = torch.randn(shape, device="cuda", dtype=torch.float16)
    vc = torch.randn(shape, device="cuda", dtype=torch.float16)
    positions = torch.tensor([0, 255, 699], device="cuda", dtype=torch.int32)
    kc2, vc2 = kc.clone(), vc.clone()
    qr = kernels.qk_norm_rope_cache(q, k, v, qw, kw, kc2, vc2, positions, inv, batch=B, tokens=1, n_heads=NH,
                                    n_kv=NK, head_dim=D, layout=layout)
    ref = kernels.attn_decode(qr, kc2, vc2, positions, batch=B, n_heads=NH, n_kv=NK, head_dim=D, max_len=S,
                              splits=1, layout=layout)
    ws = kernels.attn_decode_fused_workspace(B, NH, NK, D, splits)
    for _ in range(2):  # the second call checks that the arrival counters were reset
        out = kernels.attn_decode_fused(q, k, v, qw, kw, inv, kc, vc, positions, batch=B, n_heads=NH, n_kv=NK,
                                        head_dim=D, splits=splits, workspace=ws, layout=layout)
        torch.cuda.synchronize()
        assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
        _close(out, ref.float(), rel=2e-3, abs_=2e-3)
        if ws is not None:
            assert int(ws[-B * NH:].view(torch.int32).abs().sum()) == 0
    assert kernels.device_status() == 0


@pytest.mark.parametrize("S,pos,splits", [(16384, 16383, 8), (32768, 32767, 8), (32768, 30001, 16), (4096, 2500, 3)])
def test_attn_decode_fused_long_context(S, pos, splits):
    """Decode against 4k-32k caches (the attention sweep's decode mode): with 8 splits each CTA walks
    up to 4096 positions, i.e. 16 passes of its 8 warps over 32-position tiles; 16 splits take the
    workspace combine.  Compared with the unfused chain on the same caches."""
    from torch2vk_b200 import kernels
    from torch2vk_b200.qwen3 import Qwen3Config, inv_freq

    torch.manual_seed(S + splits)
    B, NH, NK, D = 1, 32, 8, 128
    inv = inv_freq(Qwen3Config.qwen3_8b()).cuda()
    q = torch.randn(B, NH * D, device="cuda", dtype=torch.float16)
    k = torch.randn(B, NK * D, device="cuda", dtype=torch.float16)
    v = torch.randn(B, NK * D, device="cuda", dtype=torch.float16)
    qw = 1 + 0.1 * torch.randn(D, device="cuda")
    kw = 1 + 0.1 * torch.randn(D, device="cuda")
    kc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    vc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    positions = torch.tensor([pos], device="cuda", dtype=torch.int32)
    kc2, vc2 = kc.clone(), vc.clone()
    qr = kernels.qk_norm_rope_cache(q, k, v, qw, kw, kc2, vc2, positions, inv, batch=B, tokens=1, n_heads=NH,
                                    n_kv=NK, head_dim=D)
    ref = kernels.attn_decode(qr, kc2, vc2, positions, batch=B, n_heads=NH, n_kv=NK, head_dim=D, max_len=S,
                              splits=1)
    ws = kernels.attn_decode_fused_workspace(B, NH, NK, D, splits)
    out = kernels.attn_decode_fused(q, k, v, qw, kw, inv, kc, vc, positions, batch=B, n_heads=NH, n_kv=NK,
                                    head_dim=D, splits=splits, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    _close(out, ref.float(), rel=2e-3, abs_=2e-3)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("static", [False, True])
def test_attn_decode_position_outside_cache(static):
    """A position >= max_len with an uneven split count (max_len not a multiple of splits): the kernel sets
    T2C_EINVAL in the device status, that row attends to nothing, the other rows are unaffected."""
    from torch2vk_b200 import _lib, kernels

    torch.manual_seed(4)
    B, NH, NK, D, S, splits = 3, 32, 8, 128, 700, 3
    q = torch.randn(B, NH * D, device="cuda", dtype=torch.float16)
    kc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    vc = torch.randn(B, S, NK, D, device="cuda", dtype=torch.float16)
    positions = torch.tensor([100, S, S + 40], device="cuda", dtype=torch.int32)
    kernels.device_status(clear=True)
    if static:
        out = torch.full_like(q, 7.0)
        cb, cs, ch = kernels.cache_strides(kc, "token_major")
        _lib.lib().call("t2c_attn_decode_static", _lib.ptr(q), _lib.ptr(kc), _lib.ptr(vc), _lib.ptr(out),
                        _lib.ptr(positions), B, NH, NK, D, S, cb, cs, ch, splits, _lib.stream_ptr())
    else:
        out = kernels.attn_decode(q, kc, vc, positions, batch=B, n_heads=NH, n_kv=NK, head_dim=D, max_len=S,
                                  splits=splits, out=torch.full_like(q, 7.0))
    torch.cuda.synchronize()
    assert kernels.device_status(clear=True) & (1 << 1)
    o = out.view(B, NH, D)
    _close(o[:1], _attn_ref(q.view(B, NH, D)[:1], kc[:1], vc[:1], [101], NH, NK))
    assert torch.count_nonzero(o[1:]).item() == 0


def test_attn_decode_fused_rejects_bad_arguments():
    from torch2vk_b200 import kernels
    from torch2vk_b200._lib import T2CError

    B, NH, NK, D = 1, 32, 8, 128
    t = torch.zeros(B, NH * D, device="cuda", dtype=torch.float16)
    kv = torch.zeros(B, NK * D, device="cuda", dtype=torch.float16)
    c = torch.zeros(B, 64, NK, D, device="cuda", dtype=torch.float16)
    w = torch.ones(D, device="cuda")
    pos = torch.zeros(B, device="cuda", dtype=torch.int32)
    with pytest.raises(T2CError, match="workspace"):
        kernels.attn_decode_fused(t, kv, kv, w, w, w[:64], c, c, pos, batch=B, n_heads=NH, n_kv=NK, head_dim=D,
                                  splits=12, workspace=None)
    with pytest.raises(T2CError, match="D=64"):
        kernels.attn_decode_fused(t, kv, kv, w, w, w[:64], c, c, pos, batch=B, n_heads=NH * 2, n_kv=NK * 2,
                                  head_dim=64, splits=1, workspace=None)

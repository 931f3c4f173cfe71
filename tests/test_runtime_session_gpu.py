"""The drop-in boundary on the GPU: reference-named variants dispatched through
RuntimeSession (contract validation, GGUF weight materialization, aliases,
frames) into the CUDA op table, checked against the oracle and numpy.

Tolerances: quantized linears as in test_qlinear_gpu (|err| <= 2e-3*(|ref|+rms));
fp16 elementwise / copies bit-exact; attention max-abs <= 2e-3 on O(1) values;
LM-head argmax token identical to the oracle's double-precision argmax.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

K = 512


def _tol(got, ref, rel=2e-3):
    ref = ref.astype(np.float64)
    rms = float(np.sqrt(np.mean(ref ** 2))) + 1e-30
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= rel * (np.abs(ref) + rms)), f"max err {err.max()} (rms {rms})"


@pytest.fixture(scope="module")
def model(tmp_path_factory, oracle):
    from torch2vk_b200.gguf import GGMLType, WriteTensor, write_gguf

    rng = np.random.default_rng(11)
    shapes = {"q.weight": ("q4_k", 256), "k.weight": ("q4_k", 128), "v.weight": ("q6_k", 128),
              "e.weight": ("q8_0", 64), "lm_head.weight": ("q6_k", 1000)}
    packed, tensors = {}, []
    for name, (kind, n) in shapes.items():
        w = (rng.standard_normal((n, K)) * 0.05).astype(np.float32)
        p = oracle.quantize(w, kind)
        packed[name] = (p, kind)
        tensors.append(WriteTensor(name, p, {"q4_k": GGMLType.Q4_K, "q6_k": GGMLType.Q6_K,
                                              "q8_0": GGMLType.Q8_0}[kind], (n, K)))
    emb = (rng.standard_normal((300, 1024)) * 0.05).astype(np.float32)
    packed["embed.weight"] = (oracle.quantize(emb, "q4_k"), "q4_k")
    tensors.append(WriteTensor("embed.weight", packed["embed.weight"][0], GGMLType.Q4_K, (300, 1024)))
    norm = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    tensors.append(WriteTensor("norm.weight", norm, GGMLType.F32, (K,)))
    qn = (1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    tensors.append(WriteTensor("q_norm.weight", qn, GGMLType.F32, (128,)))
    d = tmp_path_factory.mktemp("gguf")
    write_gguf(d / "model.gguf", tensors)
    return d, packed, norm, qn


def _declare(model_dir):
    from torch2vk_b200.runtime.logical import LogicalTensor, MemoryClass, TensorLifetime, TensorRole, \
        bind_logical_tensor_names
    from torch2vk_b200.runtime.types import TensorSpec, q4_k_words_layout, q6_k_halfwords_layout, \
        q8_0_halfwords_layout

    def w(key, dtype, shape, layout=None):
        kw = {} if layout is None else {"layout": layout}
        return LogicalTensor(spec=TensorSpec(dtype, shape), role=TensorRole.WEIGHT, memory=MemoryClass.MODEL_WEIGHT,
                             lifetime=TensorLifetime.MODEL, checkpoint_key=key, **kw)

    @dataclass
    class Weights:
        q: LogicalTensor
        k: LogicalTensor
        v: LogicalTensor
        e: LogicalTensor
        lm_head: LogicalTensor
        embed: LogicalTensor
        norm: LogicalTensor
        q_norm: LogicalTensor

    ws = Weights(
        q=w("q.weight", "uint32", (256, K // 256 * 36), q4_k_words_layout(logical_k=K)),
        k=w("k.weight", "uint32", (128, K // 256 * 36), q4_k_words_layout(logical_k=K)),
        v=w("v.weight", "uint16", (128, K // 256 * 105), q6_k_halfwords_layout(logical_k=K)),
        e=w("e.weight", "uint16", (64, K // 32 * 17), q8_0_halfwords_layout(logical_k=K)),
        lm_head=w("lm_head.weight", "uint16", (1000, K // 256 * 105), q6_k_halfwords_layout(logical_k=K)),
        embed=w("embed.weight", "uint32", (300, 144), q4_k_words_layout(logical_k=1024)),
        norm=w("norm.weight", "float32", (K,)),
        q_norm=w("q_norm.weight", "float32", (128,)),
    )
    bind_logical_tensor_names(ws, "model")
    return ws


def _t(name, dtype, shape, role="activation"):
    from torch2vk_b200.runtime.logical import LogicalTensor, MemoryClass, TensorLifetime, TensorRole
    from torch2vk_b200.runtime.types import TensorSpec

    r = {"activation": (TensorRole.ACTIVATION, MemoryClass.FRAME_WORKSPACE, TensorLifetime.FRAME),
         "input": (TensorRole.INPUT, MemoryClass.HOST_INPUT, TensorLifetime.FRAME),
         "state": (TensorRole.STATE, MemoryClass.REQUEST_STATE, TensorLifetime.REQUEST)}[role]
    return LogicalTensor(spec=TensorSpec(dtype, tuple(shape)), role=r[0], memory=r[1], lifetime=r[2], name=name)


def test_linears_through_session(model, oracle):
    from torch2vk_b200.runtime import variants as V
    from torch2vk_b200.runtime.session import RuntimeSession

    model_dir, packed, norm, _ = model
    ws = _declare(model_dir)
    rng = np.random.default_rng(3)
    x3 = rng.standard_normal((1, 3, K)).astype(np.float16)
    x20 = rng.standard_normal((1, 20, K)).astype(np.float16)
    res = rng.standard_normal((1, 3, 256)).astype(np.float16)
    x_in, x20_in, res_in = _t("x", "float16", x3.shape, "input"), _t("x20", "float16", x20.shape, "input"), \
        _t("res", "float16", res.shape, "input")
    rms = _t("rms", "float16", x3.shape)
    outs = {n: _t(n, "float16", (1, 3, c)) for n, c in (("yq", 256), ("yk", 128), ("yv", 128), ("ye", 64),
                                                       ("yadd", 256), ("fq", 256), ("fk", 128), ("fv", 128))}
    y20 = _t("y20", "float16", (1, 20, 128))
    with RuntimeSession.open(model_dir=model_dir, model_tensors=ws) as rt:
        rt.materialize_model_weights()
        with rt.request():
            with rt.frame("linears"):
                rt.register_host_inputs({x_in: x3, x20_in: x20, res_in: res})
                V.RMS_NORM_F32W_F32(rt, x=x_in, weight=ws.norm, output=rms)
                V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=rms, weight=ws.q, output=outs["yq"])
                V.LINEAR_NOBIAS_Q4_K_F32(rt, x=rms, weight=ws.k, output=outs["yk"])
                V.LINEAR_NOBIAS_Q6_K_MATVEC_F32(rt, x=rms, weight=ws.v, output=outs["yv"])
                V.LINEAR_NOBIAS_Q8_0_MATVEC_F32(rt, x=rms, weight=ws.e, output=outs["ye"])
                V.LINEAR_NOBIAS_Q4_K_MATVEC_ADD_F32(rt, x=rms, weight=ws.q, residual=res_in, output=outs["yadd"])
                V.LINEAR_NOBIAS_Q4_QK_Q6_V_MATVEC_F32(rt, x=rms, q_weight=ws.q, k_weight=ws.k, v_weight=ws.v,
                                                      q_output=outs["fq"], k_output=outs["fk"], v_output=outs["fv"])
                V.LINEAR_NOBIAS_Q6_K_F32(rt, x=x20_in, weight=ws.v, output=y20)
                got = {n: rt.readback(t) for n, t in outs.items()}
                got_rms = rt.readback(rms)
                got20 = rt.readback(y20)
            assert [r.shader for r in rt.dispatch_records][:2] == ["rms_norm_f32w_f32", "linear_nobias_q4_k_matvec_f32"]
    xf = x3.astype(np.float32).reshape(3, K)
    ref_rms = (xf / np.sqrt(np.mean(xf.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * norm)
    _tol(got_rms.reshape(3, K), ref_rms, rel=2e-3)
    r16 = got_rms.reshape(3, K)
    for name, key in (("yq", "q.weight"), ("yk", "k.weight"), ("yv", "v.weight"), ("ye", "e.weight"),
                      ("fq", "q.weight"), ("fk", "k.weight"), ("fv", "v.weight")):
        p, kind = packed[key]
        _tol(got[name].reshape(3, -1), oracle.matvec(p, kind, r16))
    ref_add = oracle.matvec(packed["q.weight"][0], "q4_k", r16) + res.reshape(3, 256).astype(np.float64)
    _tol(got["yadd"].reshape(3, -1), ref_add)
    _tol(got20.reshape(20, -1), oracle.matvec(packed["v.weight"][0], "q6_k", x20.reshape(20, K)))


def test_views_elementwise_and_rope(model):
    from torch2vk_b200.runtime import variants as V
    from torch2vk_b200.runtime.logical import bind_logical_tensor_alias
    from torch2vk_b200.runtime.session import RuntimeSession

    model_dir, _, _, qn = model
    ws = _declare(model_dir)
    rng = np.random.default_rng(5)
    T, H, D = 3, 2, 128
    a = rng.standard_normal((1, T, H * D)).astype(np.float16)
    b = rng.standard_normal((1, 1, H, D)).astype(np.float16)
    a_in = _t("a", "float16", a.shape, "input")
    a4 = _t("a4", "float16", (1, T, H, D))
    b_in = _t("b", "float16", b.shape, "input")
    tr = _t("tr", "float16", (1, H, T, D))
    lo, hi = _t("lo", "float16", (1, H, T, 64)), _t("hi", "float16", (1, H, T, 64))
    neg, cat = _t("neg", "float16", (1, H, T, 64)), _t("cat", "float16", (1, H, T, D))
    mulb, add4 = _t("mulb", "float16", (1, T, H, D)), _t("add4", "float16", (1, T, H, D))
    silu, mul3 = _t("silu", "float16", (1, T, H * D)), _t("mul3", "float16", (1, T, H * D))
    cos, sin = _t("cos", "float16", (1, T, D), "state"), _t("sin", "float16", (1, T, D), "state")
    nrt = _t("nrt", "float16", (1, H, T, D))
    with RuntimeSession.open(model_dir=model_dir, model_tensors=ws) as rt:
        with rt.request(state={cos: np.zeros((1, T, D), np.float16), sin: np.zeros((1, T, D), np.float16)}):
            with rt.frame("views"):
                rt.register_host_inputs({a_in: a, b_in: b})
                V.ADD_F32_18(rt, x=a_in, y=a_in, output=silu)  # warm one op, then overwrite below
                V.SILU_F32(rt, x=a_in, output=silu)
                V.MUL_F32(rt, x=silu, y=a_in, output=mul3)
                bind_logical_tensor_alias(a_in, a4)
                V.TRANSPOSE_F32(rt, x=a4, output=tr)
                V.SLICE_F32(rt, x=tr, output=lo)
                V.SLICE_F32_10(rt, x=tr, output=hi)
                V.NEG_F32(rt, x=hi, output=neg)
                V.CAT_2_F32(rt, x0=neg, x1=lo, output=cat)
                V.MUL_BROADCAST(rt, x=a4, y=b_in, output=mulb)
                V.ADD_F32(rt, x=a4, y=mulb, output=add4)
                V.ROPE_TABLE_F32(rt, start_position=7, theta=1e6, cos=cos, sin=sin)
                V.RMS_NORM_ROPE_TRANSPOSE_F16(rt, x=a4, weight=ws.q_norm, cos=cos, sin=sin, output=nrt)
                g = {n: rt.readback(t) for n, t in (("tr", tr), ("cat", cat), ("mulb", mulb), ("add4", add4),
                                                    ("silu", silu), ("mul3", mul3), ("cos", cos), ("sin", sin),
                                                    ("nrt", nrt))}
    f = np.float32
    a4n = a.reshape(1, T, H, D)
    trn = a4n.transpose(0, 2, 1, 3)
    assert np.array_equal(g["tr"], trn)
    assert np.array_equal(g["cat"], np.concatenate([(-trn[..., 64:].astype(f)).astype(np.float16), trn[..., :64]], -1))
    mb = (a4n.astype(f) * b.astype(f)).astype(np.float16)
    assert np.array_equal(g["mulb"], mb)
    assert np.array_equal(g["add4"], (a4n.astype(f) + mb.astype(f)).astype(np.float16))
    af = a.astype(np.float64)
    _tol(g["silu"], af / (1 + np.exp(-af)), rel=2e-3)
    assert np.array_equal(g["mul3"], (g["silu"].astype(f) * a.astype(f)).astype(np.float16))
    pos = 7 + np.arange(T)[:, None]
    inv = 1e6 ** (-(2.0 * (np.arange(D) % (D // 2))) / D)
    ang = pos * inv
    np.testing.assert_allclose(g["cos"][0].astype(np.float64), np.cos(ang), atol=1e-3)
    np.testing.assert_allclose(g["sin"][0].astype(np.float64), np.sin(ang), atol=1e-3)
    xn = a4n.astype(np.float64)
    xn = xn / np.sqrt(np.mean(xn ** 2, -1, keepdims=True) + 1e-6) * qn
    c, s = g["cos"].astype(np.float64)[:, :, None, :], g["sin"].astype(np.float64)[:, :, None, :]
    rot = np.concatenate([-xn[..., 64:], xn[..., :64]], -1)
    ref = (xn * c + rot * s).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(g["nrt"].astype(np.float64), ref, atol=1e-2, rtol=1e-2)


def _attn_ref(q, k, v, limit):
    """q [NH, D], k/v [NK, L, D] -> [NH, D] over positions < limit (float64)."""
    NH, D = q.shape
    NK = k.shape[0]
    out = np.zeros((NH, D))
    for h in range(NH):
        kh = h * NK // NH
        s = (k[kh, :limit] @ q[h]) / np.sqrt(D)
        p = np.exp(s - s.max())
        out[h] = (p[:, None] * v[kh, :limit]).sum(0) / p.sum()
    return out


def test_kv_cache_and_attention(model):
    from torch2vk_b200.runtime import variants as V
    from torch2vk_b200.runtime.session import RuntimeSession

    model_dir, _, _, _ = model
    ws = _declare(model_dir)
    rng = np.random.default_rng(9)
    NH, NK, D, S, T = 4, 2, 128, 64, 5
    q = (rng.standard_normal((1, NH, T, D)) / 4).astype(np.float16)
    k = (rng.standard_normal((1, NK, T, D)) / 4).astype(np.float16)
    v = rng.standard_normal((1, NK, T, D)).astype(np.float16)
    q_in, k_in, v_in = (_t(n, "float16", x.shape, "input") for n, x in (("q", q), ("k", k), ("v", v)))
    pos_in = _t("pos", "int64", (T,), "input")
    kc, vc = _t("kc", "float16", (1, NK, S, D), "state"), _t("vc", "float16", (1, NK, S, D), "state")
    causal = _t("causal", "float16", (1, NH, T, D))
    q1 = _t("q1", "float16", (1, NH, 1, D), "input")
    k1, v1 = _t("k1", "float16", (1, NK, 1, D), "input"), _t("v1", "float16", (1, NK, 1, D), "input")
    dec = _t("dec", "float16", (1, NH, 1, D))
    qd = (rng.standard_normal((1, NH, 1, D)) / 4).astype(np.float16)
    kd = (rng.standard_normal((1, NK, 1, D)) / 4).astype(np.float16)
    vd = rng.standard_normal((1, NK, 1, D)).astype(np.float16)
    # token-major fused write + attend
    ktm, vtm = _t("ktm", "float16", (1, S, NK, D), "state"), _t("vtm", "float16", (1, S, NK, D), "state")
    v1tm = _t("v1tm", "float16", (1, 1, NK, D), "input")
    dec2 = _t("dec2", "float16", (1, NH, 1, D))
    zeros = np.zeros((1, NK, S, D), np.float16)
    base_tm = rng.standard_normal((1, S, NK, D)).astype(np.float16)
    with RuntimeSession.open(model_dir=model_dir, model_tensors=ws) as rt:
        with rt.request(state={kc: zeros, vc: zeros, ktm: base_tm, vtm: base_tm}):
            with rt.frame("prefill"):
                rt.register_host_inputs({q_in: q, k_in: k, v_in: v, pos_in: np.arange(T, dtype=np.int64)})
                V.KV_CACHE_WRITE_F16(rt, cache=kc, cache_position=pos_in, src=k_in)
                V.KV_CACHE_WRITE_F16(rt, cache=vc, cache_position=pos_in, src=v_in)
                V.SDPA_CAUSAL_F32(rt, q=q_in, k=k_in, v=v_in, output=causal)
                got_causal = rt.readback(causal)
            with rt.frame("decode"):
                rt.register_host_inputs({q1: qd, k1: kd, v1: vd, v1tm: vd.transpose(0, 2, 1, 3).copy()})
                V.KV_CACHE_WRITE_DECODE_F16(rt, cache=kc, src=k1, cache_position=T)
                V.KV_CACHE_WRITE_DECODE_F16(rt, cache=vc, src=v1, cache_position=T)
                V.SDPA_DECODE_CACHE_F16(rt, q=q1, k=kc, v=vc, output=dec, cache_position=T)
                V.SDPA_DECODE_CACHE_WRITE_F32(rt, q=q1, new_k=k1, new_v=v1tm, k_cache=ktm, v_cache=vtm, output=dec2,
                                              cache_position=9)
                got_dec, got_dec2 = rt.readback(dec), rt.readback(dec2)
                got_kc, got_ktm = rt.readback(kc), rt.readback(ktm)
    assert np.array_equal(got_kc[0, :, :T], k[0])
    assert np.array_equal(got_kc[0, :, T], kd[0, :, 0])
    assert np.array_equal(got_ktm[0, 9], kd[0, :, 0])
    assert np.array_equal(got_ktm[0, 8], base_tm[0, 8])
    for t in range(T):
        ref = _attn_ref(q[0, :, t].astype(np.float64), k[0].astype(np.float64), v[0].astype(np.float64), t + 1)
        np.testing.assert_allclose(got_causal[0, :, t].astype(np.float64), ref, atol=2e-3)
    kfull = np.concatenate([k[0], kd[0]], 1).astype(np.float64)
    vfull = np.concatenate([v[0], vd[0]], 1).astype(np.float64)
    np.testing.assert_allclose(got_dec[0, :, 0].astype(np.float64),
                               _attn_ref(qd[0, :, 0].astype(np.float64), kfull, vfull, T + 1), atol=2e-3)
    ktm_ref = base_tm[0].transpose(1, 0, 2).astype(np.float64).copy()
    vtm_ref = ktm_ref.copy()
    ktm_ref[:, 9], vtm_ref[:, 9] = kd[0, :, 0], vd[0, :, 0]
    np.testing.assert_allclose(got_dec2[0, :, 0].astype(np.float64),
                               _attn_ref(qd[0, :, 0].astype(np.float64), ktm_ref, vtm_ref, 10), atol=2e-3)


def test_embedding_lm_head_select_store(model, oracle):
    from torch2vk_b200.runtime import variants as V
    from torch2vk_b200.runtime.session import RuntimeSession

    model_dir, packed, _, _ = model
    ws = _declare(model_dir)
    rng = np.random.default_rng(13)
    ids = rng.integers(0, 300, size=(1, 4)).astype(np.int64)
    ids_in = _t("ids", "int64", ids.shape, "input")
    emb = _t("emb", "float16", (1, 4, 1024))
    x = rng.standard_normal((1, 1, K)).astype(np.float16)
    x_in = _t("x", "float16", x.shape, "input")
    G, C = 250, 1
    ps, pt = _t("ps", "float32", (G,)), _t("pt", "uint32", (G,))
    cs, ct = _t("cs", "float32", (C,)), _t("ct", "uint32", (C,))
    eos_in = _t("eos", "int64", (2,), "input")
    nt, done = _t("nt", "int64", (1, 1), "state"), _t("done", "uint32", (1,), "state")
    gen, glen, stop = _t("gen", "int64", (1, 8), "state"), _t("glen", "uint32", (1,), "state"), \
        _t("stop", "uint32", (1,), "state")
    with RuntimeSession.open(model_dir=model_dir, model_tensors=ws) as rt:
        with rt.request(state={nt: np.zeros((1, 1), np.int64), done: np.zeros(1, np.uint32),
                               gen: np.zeros((1, 8), np.int64), glen: np.zeros(1, np.uint32),
                               stop: np.zeros(1, np.uint32)}):
            with rt.frame("head"):
                rt.register_host_inputs({ids_in: ids, x_in: x, eos_in: np.array([998, 999], np.int64)})
                V.EMBEDDING_Q4_K_F32(rt, weight=ws.embed, indices=ids_in, output=emb)
                V.LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16(rt, x=x_in, weight=ws.lm_head, partial_scores=ps, partial_tokens=pt)
                V.QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32(rt, scores=ps, tokens=pt, chunk_scores=cs, chunk_tokens=ct)
                V.QWEN3_TOKEN_SELECT_REDUCE_F32(rt, partial_scores=cs, partial_tokens=ct, eos_token_ids=eos_in,
                                                next_token=nt, done=done)
                V.QWEN3_TOKEN_STORE_EOS(rt, next_token=nt, done=done, generated_tokens=gen, generated_length=glen,
                                        stopped=stop, token_index=2)
                got_emb = rt.readback(emb)
            got_nt = int(rt.read_request_state(nt).reshape(-1)[0])
            got_gen = rt.read_request_state(gen)
            got_len = int(rt.read_request_state(glen)[0])
    deq = oracle.dequantize_np(packed["embed.weight"][0], "q4_k", 1024)
    assert np.array_equal(got_emb[0], deq[ids[0]].astype(np.float16))
    scores = oracle.matvec(packed["lm_head.weight"][0], "q6_k", x.reshape(1, K))[0]
    assert got_nt == int(np.argmax(scores))
    assert got_gen[0, 2] == got_nt and got_len == 3


def test_dispatch_outside_frame_and_missing_weight_key(model):
    from torch2vk_b200.runtime import variants as V
    from torch2vk_b200.runtime.session import RuntimeSession

    model_dir, _, _, _ = model
    ws = _declare(model_dir)
    x_in = _t("x", "float16", (1, 1, K), "input")
    y = _t("y", "float16", (1, 1, 256))
    with RuntimeSession.open(model_dir=model_dir, model_tensors=ws) as rt:
        with pytest.raises(RuntimeError, match="active rt.frame"):
            V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=x_in, weight=ws.q, output=y)
        with rt.frame("bad"):
            with pytest.raises(ValueError, match="expects dtype"):
                V.LINEAR_NOBIAS_Q6_K_MATVEC_F32(rt, x=x_in, weight=ws.q, output=y)


def test_replay_plans(model, oracle):
    """rt.build_replay_plan / execute_replay (src/torch2vk/runtime/replay.py:226-364): a frame without
    push-constant inputs replays from a CUDA graph (first execution captures it) and picks up new step
    inputs staged with stage_replay_step_inputs; a decode frame replays with a new cache_position."""
    from torch2vk_b200.runtime import variants as V
    from torch2vk_b200.runtime.replay import execute_replay, stage_replay_step_inputs
    from torch2vk_b200.runtime.session import RuntimeSession

    model_dir, packed, norm, _ = model
    ws = _declare(model_dir)
    rng = np.random.default_rng(12)
    x_in = _t("xr", "float16", (1, 3, K), "input")
    rms, yq = _t("rmsr", "float16", (1, 3, K)), _t("yqr", "float16", (1, 3, 256))
    xs = [rng.standard_normal((1, 3, K)).astype(np.float16) for _ in range(3)]
    NH, NK, D, S, T = 4, 2, 128, 64, 5
    q1 = _t("q1r", "float16", (1, NH, 1, D), "input")
    k1, v1 = _t("k1r", "float16", (1, NK, 1, D), "input"), _t("v1r", "float16", (1, NK, 1, D), "input")
    kc, vc = _t("kcr", "float16", (1, NK, S, D), "state"), _t("vcr", "float16", (1, NK, S, D), "state")
    dec = _t("decr", "float16", (1, NH, 1, D))
    kbase = (rng.standard_normal((1, NK, S, D)) / 4).astype(np.float16)
    vbase = rng.standard_normal((1, NK, S, D)).astype(np.float16)
    qd = (rng.standard_normal((1, NH, 1, D)) / 4).astype(np.float16)
    kd = (rng.standard_normal((1, NK, 1, D)) / 4).astype(np.float16)
    vd = rng.standard_normal((1, NK, 1, D)).astype(np.float16)
    with RuntimeSession.open(model_dir=model_dir, model_tensors=ws) as rt:
        rt.materialize_model_weights()
        with rt.request(state={kc: kbase, vc: vbase}):
            with rt.frame("lin"):
                rt.register_host_inputs({x_in: xs[0]})
                V.RMS_NORM_F32W_F32(rt, x=x_in, weight=ws.norm, output=rms)
                V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=rms, weight=ws.q, output=yq)
                first = rt.readback(yq)
            plan = rt.build_replay_plan(name="lin", frame="lin", readback_tensors={"y": yq})
            assert plan.dynamic_push_constant_names == ()
            outs = []
            for x in xs:  # execution 1 captures the graph, 2 and 3 replay it
                stage_replay_step_inputs(rt, plan=plan, inputs={x_in: x})
                outs.append(np.frombuffer(execute_replay(plan)["y"], np.float16).reshape(1, 3, 256))
            assert plan.graph is not None
            with rt.frame("dec"):
                rt.register_host_inputs({q1: qd, k1: kd, v1: vd})
                V.KV_CACHE_WRITE_DECODE_F16(rt, cache=kc, src=k1, cache_position=T)
                V.KV_CACHE_WRITE_DECODE_F16(rt, cache=vc, src=v1, cache_position=T)
                V.SDPA_DECODE_CACHE_F16(rt, q=q1, k=kc, v=vc, output=dec, cache_position=T)
            dplan = rt.build_replay_plan(name="dec", frame="dec", readback_tensors={"dec": dec})
            assert dplan.dynamic_push_constant_names == ("cache_position",)
            got = np.frombuffer(execute_replay(dplan, dynamic_push_constants={"cache_position": T + 3})["dec"],
                                np.float16).reshape(1, NH, 1, D)
            got_kc = rt.readback(kc)
    assert np.array_equal(outs[0], first)
    for x, out in zip(xs, outs):
        xf = x.astype(np.float32).reshape(3, K)
        r16 = (xf / np.sqrt(np.mean(xf.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * norm).astype(np.float16)
        _tol(out.reshape(3, -1), oracle.matvec(packed["q.weight"][0], "q4_k", r16), rel=4e-3)
    assert np.array_equal(got_kc[0, :, T], kd[0, :, 0]) and np.array_equal(got_kc[0, :, T + 3], kd[0, :, 0])
    kfull, vfull = kbase[0].astype(np.float64).copy(), vbase[0].astype(np.float64).copy()
    for p in (T, T + 3):
        kfull[:, p], vfull[:, p] = kd[0, :, 0], vd[0, :, 0]
    np.testing.assert_allclose(got[0, :, 0].astype(np.float64),
                               _attn_ref(qd[0, :, 0].astype(np.float64), kfull, vfull, T + 4), atol=2e-3)


def test_replay_plan_dynamic_graph(model):
    """A decode frame whose ops take dynamic push constants (rope start_position / theta, cache_position,
    token_index) is captured into a CUDA graph after its first execution; later steps replay the graph
    with the values written to device slots (src/torch2vk/runtime/replay.py:226-364), and a step that
    changes a baked value (theta) runs the dispatches directly."""
    from torch2vk_b200.runtime import variants as V
    from torch2vk_b200.runtime.replay import execute_replay, stage_replay_step_inputs
    from torch2vk_b200.runtime.session import RuntimeSession

    model_dir = model[0]
    ws = _declare(model_dir)
    NH, NK, D, S, P, G = 4, 2, 128, 640, 300, 8
    rng = np.random.default_rng(21)
    q1 = _t("q1g", "float16", (1, NH, 1, D), "input")
    k1, v1 = _t("k1g", "float16", (1, NK, 1, D), "input"), _t("v1g", "float16", (1, NK, 1, D), "input")
    v1t = _t("v1tg", "float16", (1, 1, NK, D), "input")
    nt, dn = _t("ntg", "int64", (1, 1), "input"), _t("dng", "uint32", (1,), "input")
    kc, vc = _t("kcg", "float16", (1, NK, S, D), "state"), _t("vcg", "float16", (1, NK, S, D), "state")
    kt, vt = _t("ktg", "float16", (1, S, NK, D), "state"), _t("vtg", "float16", (1, S, NK, D), "state")
    gen = _t("geng", "int64", (1, G), "state")
    glen, stp = _t("glg", "uint32", (1,), "state"), _t("stg", "uint32", (1,), "state")
    dec, dec2 = _t("decg", "float16", (1, NH, 1, D)), _t("dec2g", "float16", (1, NH, 1, D))
    cos, sin = _t("cosg", "float16", (1, 1, D)), _t("sing", "float16", (1, 1, D))
    kbase = (rng.standard_normal((1, NK, S, D)) / 4).astype(np.float16)
    vbase = rng.standard_normal((1, NK, S, D)).astype(np.float16)
    qd = (rng.standard_normal((1, NH, 1, D)) / 4).astype(np.float16)
    steps = [((rng.standard_normal((1, NK, 1, D)) / 4).astype(np.float16),
              rng.standard_normal((1, NK, 1, D)).astype(np.float16)) for _ in range(5)]

    def step_inputs(j):
        kd, vd = steps[j]
        return {q1: qd, k1: kd, v1: vd, v1t: vd.transpose(0, 2, 1, 3).copy(),
                nt: np.array([[1000 + j]], np.int64), dn: np.zeros(1, np.uint32)}

    def cos_ref(p, theta):
        inv = theta ** (-2.0 * (np.arange(D) % (D // 2)) / D)
        return np.cos(p * inv)

    zeros = {gen: np.zeros((1, G), np.int64), glen: np.zeros(1, np.uint32), stp: np.zeros(1, np.uint32)}
    with RuntimeSession.open(model_dir=model_dir, model_tensors=ws) as rt:
        rt.materialize_model_weights()
        state = {kc: kbase, vc: vbase, kt: kbase.transpose(0, 2, 1, 3).copy(),
                 vt: vbase.transpose(0, 2, 1, 3).copy(), **zeros}
        with rt.request(state=state):
            with rt.frame("step"):
                rt.register_host_inputs(step_inputs(0))
                V.ROPE_TABLE_F32(rt, cos=cos, sin=sin, start_position=P, theta=1e6)
                V.KV_CACHE_WRITE_DECODE_F16(rt, cache=kc, src=k1, cache_position=P)
                V.KV_CACHE_WRITE_DECODE_F16(rt, cache=vc, src=v1, cache_position=P)
                V.SDPA_DECODE_CACHE_F16(rt, q=q1, k=kc, v=vc, output=dec, cache_position=P)
                V.SDPA_DECODE_CACHE_WRITE_F32(rt, q=q1, new_k=k1, new_v=v1t, k_cache=kt, v_cache=vt, output=dec2,
                                              cache_position=P)
                V.QWEN3_TOKEN_STORE_EOS(rt, next_token=nt, done=dn, generated_tokens=gen, generated_length=glen,
                                        stopped=stp, token_index=0)
            plan = rt.build_replay_plan(name="step", frame="step",
                                        readback_tensors={"dec": dec, "dec2": dec2, "cos": cos})
            assert set(plan.dynamic_push_constant_names) == {"cache_position", "start_position", "theta",
                                                             "token_index"}
            outs = []
            for j in range(1, 5):  # step 1 runs directly and captures; steps 2-4 replay the graph
                stage_replay_step_inputs(rt, plan=plan, inputs=step_inputs(j))
                r = execute_replay(plan, dynamic_push_constants={"cache_position": P + j, "start_position": P + j,
                                                                 "theta": 1e6, "token_index": j})
                outs.append({n: np.frombuffer(v, np.float16) for n, v in r.items()})
            assert plan.graph is not None and plan.push_slots is not None
            assert (plan.direct_executions, plan.graph_replays) == (1, 3)
            r = execute_replay(plan, dynamic_push_constants={"cache_position": P + 4, "start_position": P + 4,
                                                             "theta": 1e4, "token_index": 4})
            assert (plan.direct_executions, plan.graph_replays) == (2, 3)
            cos_1e4 = np.frombuffer(r["cos"], np.float16)
            got_kc, got_kt, got_gen = rt.readback(kc), rt.readback(kt), rt.readback(gen)
    kfull, vfull = kbase[0].astype(np.float64).copy(), vbase[0].astype(np.float64).copy()
    kfull[:, P], vfull[:, P] = steps[0][0][0, :, 0], steps[0][1][0, :, 0]
    for j, o in enumerate(outs, start=1):
        p = P + j
        kfull[:, p], vfull[:, p] = steps[j][0][0, :, 0], steps[j][1][0, :, 0]
        ref = _attn_ref(qd[0, :, 0].astype(np.float64), kfull, vfull, p + 1)
        np.testing.assert_allclose(o["dec"].reshape(NH, D), ref, atol=2e-3)
        np.testing.assert_allclose(o["dec2"].reshape(NH, D), ref, atol=2e-3)
        np.testing.assert_allclose(o["cos"].astype(np.float64), cos_ref(p, 1e6), atol=2e-3)
    np.testing.assert_allclose(cos_1e4.astype(np.float64), cos_ref(P + 4, 1e4), atol=2e-3)
    for j in range(5):
        assert np.array_equal(got_kc[0, :, P + j], steps[j][0][0, :, 0])
        assert np.array_equal(got_kt[0, P + j], steps[j][0][0, :, 0])
    assert np.array_equal(got_kc[0, :, :P], kbase[0, :, :P]) and np.array_equal(got_kc[0, :, P + 5:], kbase[0, :, P + 5:])
    assert got_gen[0, :5].tolist() == [1000, 1001, 1002, 1003, 1004]


def test_session_decode_plan_matches_direct_frames(tmp_path):
    """A Qwen3-shaped decode step through the session (torch2vk_b200.qwen3_session: the optimized
    variants of src/models/optimized_qwen3/dispatch/decode_layer.py:36-128 and the greedy head) gives
    bit-identical next-token scores and tokens whether each step is dispatched as a frame or replayed
    from the captured graph of a replay plan."""
    from torch2vk_b200.qwen3_session import SessionDecodeModel
    from torch2vk_b200.runtime.replay import execute_replay, stage_replay_step_inputs
    from torch2vk_b200.runtime.session import RuntimeSession

    m = SessionDecodeModel(layers=2, vocab=4096, max_seq=256, seed=3)
    m.write_gguf(tmp_path)
    rng = np.random.default_rng(4)
    xs = [(rng.standard_normal((1, 1, m.hidden)) * 0.5).astype(np.float16) for _ in range(6)]
    eos = np.array([4094, 4095], np.int64)
    start = 40
    with RuntimeSession.open(model_dir=tmp_path, model_tensors=m.weights) as rt:
        rt.materialize_model_weights()
        with rt.request(state=m.request_state()):
            direct = []
            for j in range(6):
                with rt.frame(f"d{j}"):
                    rt.register_host_inputs({m.x_in: xs[j], m.eos: eos})
                    m.step(rt, start + j, j)
                    direct.append((rt.readback(m.cs), rt.readback(m.next_token)))
            gen_direct = rt.readback(m.generated)
        with rt.request(state=m.request_state()):
            with rt.frame("f0"):
                rt.register_host_inputs({m.x_in: xs[0], m.eos: eos})
                m.step(rt, start, 0)
            plan = rt.build_replay_plan(name="decode", frame="f0",
                                        readback_tensors={"cs": m.cs, "next": m.next_token})
            replayed = []
            for j in range(1, 6):
                stage_replay_step_inputs(rt, plan=plan, inputs={m.x_in: xs[j], m.eos: eos})
                r = execute_replay(plan, dynamic_push_constants={"cache_position": start + j,
                                                                 "start_position": start + j, "theta": 1e6,
                                                                 "token_index": j})
                replayed.append((np.frombuffer(r["cs"], np.float32), np.frombuffer(r["next"], np.int64)))
            gen_replay = rt.readback(m.generated)
    assert (plan.direct_executions, plan.graph_replays) == (1, 4)
    for (cs_d, nt_d), (cs_r, nt_r) in zip(direct[1:], replayed):
        assert np.array_equal(cs_d.reshape(-1), cs_r) and np.array_equal(nt_d.reshape(-1), nt_r)
    assert np.array_equal(gen_direct[0, :6], gen_replay[0, :6])

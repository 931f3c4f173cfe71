"""Qwen3-ASR audio encoder kernels on the GPU against fp32 torch / the CPU oracle."""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel_close(got, ref, rel=4e-3):
    """|got - ref| <= rel * (|ref| + rms(ref)): the tensor-core bound (fp16 operands) used for the GEMMs."""
    got, ref = got.float().cpu(), ref.float().cpu()
    rms = ref.pow(2).mean().sqrt()
    err = (got - ref).abs()
    bound = rel * (ref.abs() + rms)
    assert bool((err <= bound).all()), f"max err {float(err.max())}, bound there {float(bound.flatten()[err.argmax()])}"


def _q8(oracle, w: np.ndarray):
    """Q8_0 rows (K padded to 32) on the GPU and the dequantized fp32 weight of the original shape."""
    from oracle.asr_ref import q8_rows

    rows = q8_rows(w)
    packed = oracle.quantize(rows, "q8_0")
    deq = oracle.dequantize(packed, "q8_0", rows.shape[1])[:, :int(np.prod(w.shape[1:]))].reshape(w.shape)
    return torch.from_numpy(packed).cuda(), torch.from_numpy(deq.astype(np.float32))


@pytest.mark.parametrize("m,n,k,bias,gelu", [(1, 96, 128, True, False), (33, 896, 896, True, False),
                                            (130, 3584, 896, True, True), (70, 100, 7680, False, False),
                                            (5, 64, 40, True, True), (390, 5120, 1280, True, True),
                                            (390, 1280, 5120, True, False), (33, 1300, 1280, True, False)])
def test_linear_q8_0_bias(oracle, m, n, k, bias, gelu):
    """K a multiple of 256 and more than 4 rows: the tcgen05 GEMM with the bias / GELU epilogue
    (the encoder's d_model 1280 and FFN 5120 shapes); otherwise the mma.sync Q8_0 GEMM."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(m + n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    wq, wd = _q8(oracle, w)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float16))
    b = torch.from_numpy((rng.standard_normal(n) * 0.1).astype(np.float32)) if bias else None
    y = kernels.linear_q8_0_bias(x.cuda(), wq, b.cuda() if bias else None, n, gelu=gelu)
    ref = x.float() @ wd.T + (b if bias else 0.0)
    if gelu:
        ref = F.gelu(ref)
    _rel_close(y, ref)


@pytest.mark.parametrize("b,ci,h,w,co", [(3, 1, 128, 100, 32), (2, 32, 64, 50, 48), (1, 24, 17, 9, 40)])
def test_conv2d_q8_0(oracle, b, ci, h, w, co):
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(ci * co + h)
    wt = (rng.standard_normal((co, ci, 3, 3)) * 0.1).astype(np.float32)
    wq, wd = _q8(oracle, wt)
    bias = torch.from_numpy((rng.standard_normal(co) * 0.1).astype(np.float32))
    x = torch.from_numpy(rng.standard_normal((b, ci, h, w)).astype(np.float16))
    y = kernels.conv2d_q8_0(x.cuda(), wq, bias.cuda(), co, gelu=True)
    ref = F.gelu(F.conv2d(x.float(), wd, bias, stride=2, padding=1))
    assert y.shape == ref.shape
    _rel_close(y, ref)
    # the channels-last output holds the same values
    ycl = kernels.conv2d_q8_0(x.cuda(), wq, bias.cuda(), co, gelu=True, channels_last_out=True)
    assert torch.equal(ycl.permute(0, 3, 1, 2), y)


@pytest.mark.parametrize("b,ci,h,w,co,nhwc", [(2, 40, 16, 20, 48, False), (2, 40, 16, 20, 48, True),
                                               (1, 480, 32, 25, 480, True), (3, 32, 9, 7, 136, False)])
def test_conv_as_im2col_gemm(oracle, b, ci, h, w, co, nhwc):
    """The tower's 480-channel convolutions: im2col (NCHW or NHWC input through strides, K padded to a
    multiple of 256 with zeros) and the tcgen05 Q8_0 GEMM with bias + GELU, against F.conv2d on the
    dequantized weights."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(ci * co + h + int(nhwc))
    wt = (rng.standard_normal((co, ci, 3, 3)) * 0.05).astype(np.float32)
    k = ci * 9
    kp = (k + 255) // 256 * 256
    rows = np.concatenate([wt.reshape(co, k), np.zeros((co, kp - k), np.float32)], axis=1)
    wq = torch.from_numpy(oracle.quantize(rows, "q8_0")).cuda()
    wd = torch.from_numpy(oracle.dequantize(oracle.quantize(rows, "q8_0"), "q8_0", kp)[:, :k].reshape(co, ci, 3, 3))
    bias = torch.from_numpy((rng.standard_normal(co) * 0.1).astype(np.float32))
    x = torch.from_numpy(rng.standard_normal((b, ci, h, w)).astype(np.float16))
    xg = x.cuda().permute(0, 2, 3, 1).contiguous() if nhwc else x.cuda()
    sb, s1, s2, s3 = xg.stride()
    strides = (sb, s3, s1, s2) if nhwc else (sb, s1, s2, s3)
    cols = kernels.im2col(xg, channels=ci, height=h, width=w, strides_bchw=strides, batch=b, kp=kp,
                          channels_last=nhwc)
    if nhwc:  # the 16-byte channel gathers give the same columns as the strided element path
        assert torch.equal(cols, kernels.im2col(xg, channels=ci, height=h, width=w, strides_bchw=strides, batch=b,
                                                kp=kp))
    ho, wo = (h - 1) // 2 + 1, (w - 1) // 2 + 1
    assert cols.shape == (b * ho * wo, kp)
    assert torch.count_nonzero(cols[:, k:]) == 0
    y = kernels.linear_q8_0_bias(cols, wq, bias.cuda(), co, gelu=True).view(b, ho, wo, co).permute(0, 3, 1, 2)
    ref = F.gelu(F.conv2d(x.float(), wd, bias, stride=2, padding=1))
    assert y.shape == ref.shape
    _rel_close(y.contiguous(), ref)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("rows,cols", [(33, 896), (1, 128), (7, 4096)])
def test_layer_norm(rows, cols):
    from torch2vk_b200 import kernels

    torch.manual_seed(rows)
    x = (torch.randn(rows, cols) * 2 + 0.5).half()
    w, b = torch.rand(cols) + 0.5, torch.randn(cols) * 0.1
    y = kernels.layer_norm(x.cuda(), w.cuda(), b.cuda(), 1e-5)
    ref = F.layer_norm(x.float(), (cols,), w, b, 1e-5)
    assert float((y.float().cpu() - ref).abs().max()) <= 2e-3 * (1 + float(ref.abs().max()))


def test_gelu_and_index_rows():
    from torch2vk_b200 import kernels

    x = torch.randn(5, 37, 96).half()
    y = kernels.gelu(x.cuda())
    assert float((y.float().cpu() - F.gelu(x.float())).abs().max()) <= 2e-3
    table = torch.randn(20, 48).half().cuda()
    idx = torch.tensor([3, 0, 19, 3, 7], dtype=torch.int64).cuda()
    assert torch.equal(kernels.index_rows(table, idx), table[idx])
    assert kernels.device_status() == 0
    kernels.index_rows(table, torch.tensor([1, 20], dtype=torch.int64).cuda())
    torch.cuda.synchronize()
    assert kernels.device_status() != 0  # out-of-range index reported, not read


@pytest.mark.parametrize("t,windows", [(33, [26, 7]), (390, [104, 104, 104, 78]), (70, [70])])
def test_attn_masked_windows(t, windows):
    from torch2vk_b200 import kernels

    torch.manual_seed(t)
    H, D = 3, 64
    q, k, v = (torch.randn(1, H, t, D).half() for _ in range(3))
    mask = torch.full((1, 1, t, t), float("-inf"))
    a = 0
    for wlen in windows:
        mask[0, 0, a:a + wlen, a:a + wlen] = 0.0
        a += wlen
    out = kernels.attn_masked(q.cuda(), k.cuda(), v.cuda(), mask.half().cuda(), scale=1 / math.sqrt(D))
    s = q.float() @ k.float().transpose(-1, -2) / math.sqrt(D) + mask
    ref = torch.softmax(s, -1) @ v.float()
    assert float((out.float().cpu() - ref).abs().max()) <= 2e-3


def test_asr_encoder_matches_oracle(oracle):
    """The encoder (tiny configuration, Q8_0 weights, fp16 activations) against the fp32 oracle run on
    the same dequantized weights: cosine >= 0.999 and max |err| <= 2e-2 * max |ref| (layer-output bar)."""
    from oracle import asr_ref
    from test_asr_cpu import TINY, _golden
    from torch2vk_b200.asr import AsrEncoderRunner, prepare_inputs, quantized_names

    g, mel, params = _golden()
    inputs = prepare_inputs(mel, TINY)
    runner = AsrEncoderRunner(TINY, params)
    out = runner.forward(runner.upload(inputs)).float().cpu().numpy()
    ref = asr_ref.encoder_forward(
        asr_ref.dequantized_params(params, quantized_names(TINY), oracle.quantize, oracle.dequantize), inputs, TINY)
    cos = float((out * ref).sum() / (np.linalg.norm(out) * np.linalg.norm(ref)))
    assert cos >= 0.999, cos
    assert float(np.abs(out - ref).max()) <= 2e-2 * float(np.abs(ref).max())
    # and close to the reference module's own (unquantized fp32) output
    golden = g["golden"]
    assert float((out * golden).sum() / (np.linalg.norm(out) * np.linalg.norm(golden))) >= 0.99
    from torch2vk_b200 import kernels
    assert kernels.device_status() == 0


def test_text_decoder_embedding_and_audio_inject(oracle):
    """ExportEmbeddingQ8_0Program (fp16 of d * q, exact against the oracle decoder) and
    ExportIndexCopyF32Program (row scatter, exact; an out-of-range row is skipped and reported)."""
    from torch2vk_b200 import kernels

    rng = np.random.default_rng(4)
    vocab, h = 500, 1024
    packed = oracle.quantize((rng.standard_normal((vocab, h)) * 0.05).astype(np.float32), "q8_0")
    table = oracle.dequantize(packed, "q8_0", h).astype(np.float16)
    ids = np.array([[3, 499, 0, 3, 250, 17]], np.int64)
    out = kernels.embedding_q8_0(torch.from_numpy(packed).cuda(), torch.from_numpy(ids).cuda(), h, vocab)
    assert np.array_equal(out.cpu().numpy(), table[ids])

    B, T, S = 1, 40, 12
    cache = rng.standard_normal((B, T, h)).astype(np.float16)
    src = rng.standard_normal((B, S, h)).astype(np.float16)
    index = np.arange(5, 5 + S, dtype=np.int64)
    dev = torch.from_numpy(cache.copy()).cuda()
    kernels.device_status(clear=True)
    kernels.index_copy_rows(dev, torch.from_numpy(index).cuda(), torch.from_numpy(src).cuda())
    want = cache.copy()
    want[:, index] = src
    assert np.array_equal(dev.cpu().numpy(), want)
    assert kernels.device_status(clear=True) == 0
    bad = index.copy()
    bad[3] = T + 2
    dev = torch.from_numpy(cache.copy()).cuda()
    kernels.index_copy_rows(dev, torch.from_numpy(bad).cuda(), torch.from_numpy(src).cuda())
    want = cache.copy()
    keep = np.arange(S) != 3
    want[:, bad[keep]] = src[:, keep]
    assert np.array_equal(dev.cpu().numpy(), want)
    assert kernels.device_status(clear=True) & (1 << 1)


def test_rope_table_f32_and_quantize_ops(oracle):
    """RopeTableOutputF32Program (fp32 table; its fp16 rounding equals the fp16 table) and the GGUF
    quantizer programs through the op table (bit-exact with the oracle)."""
    from types import SimpleNamespace

    from torch2vk_b200 import kernels
    from torch2vk_b200.runtime import optable

    c32, s32 = torch.empty(2, 33, 128, device="cuda"), torch.empty(2, 33, 128, device="cuda")
    c16, s16 = (torch.empty(2, 33, 128, dtype=torch.float16, device="cuda") for _ in range(2))
    v = SimpleNamespace(name="rope_table_output_f32", contract=SimpleNamespace(class_name="RopeTableOutputF32Program"))
    optable.OPS["RopeTableOutputF32Program"](None, v, {"cos": c32, "sin": s32}, {},
                                             {"theta": 1e6, "start_position": 1000, "attention_scaling": 1.0})
    kernels.rope_table(c16, s16, theta=1e6, start_position=1000)
    assert torch.equal(c32.half(), c16) and torch.equal(s32.half(), s16)
    pos = 1000 + np.arange(33, dtype=np.float64)
    inv = 1e6 ** (-(2 * (np.arange(128) % 64)) / 128)
    assert np.abs(c32[0].cpu().numpy() - np.cos(pos[:, None] * inv[None, :])).max() < 2e-3

    rng = np.random.default_rng(9)
    for cls, kind, dtype, words in (("GGUFQuantizeQ4KF32Program", "q4_k", torch.int32, 36),
                                    ("GGUFQuantizeQ6KF32Program", "q6_k", torch.int16, 105),
                                    ("GGUFQuantizeQ8_0F32Program", "q8_0", torch.int16, 17 * 8)):
        x = (rng.standard_normal((24, 256)) * 0.1).astype(np.float32)
        out = torch.empty(24, words, dtype=dtype, device="cuda")
        v = SimpleNamespace(name=cls, contract=SimpleNamespace(class_name=cls))
        optable.OPS[cls](None, v, {"x": torch.from_numpy(x).cuda(), "output": out}, {"R": 24, "K": 256}, {})
        assert np.array_equal(out.cpu().numpy().view(np.uint8).reshape(24, -1), oracle.quantize(x, kind)), cls


def test_large_cache_write_and_rope_table():
    """Launches above the surface helper's grid cap (148 x 64 blocks of 256 threads): a 4096-token
    head-major cache write (8 heads x 128, 4.2M elements, kv_cache_write_f16.py:22-92) and a rope table
    of 2 x 10000 x 128 entries write every element; the table with its start read from device memory
    equals the host-start one."""
    from torch2vk_b200 import kernels

    B, H, T, D, S = 1, 8, 4096, 128, 4160
    gen = torch.Generator(device="cuda").manual_seed(5)
    src = torch.randn(B, H, T, D, device="cuda", generator=gen).half()
    cache = torch.zeros(B, H, S, D, dtype=torch.float16, device="cuda")
    pos = torch.arange(40, 40 + T, dtype=torch.int64, device="cuda")
    kernels.kv_cache_write(cache, src, cache_strides_bsh=(H * S * D, D, S * D), seq_len=S,
                           src_strides_bth=(H * T * D, D, T * D), batch=B, heads=H, tokens=T, head_dim=D, positions=pos)
    assert torch.equal(cache[:, :, 40:40 + T], src) and not cache[:, :, :40].any() and not cache[:, :, 40 + T:].any()
    cache.zero_()
    kernels.kv_cache_write(cache, src, cache_strides_bsh=(H * S * D, D, S * D), seq_len=S,
                           src_strides_bth=(H * T * D, D, T * D), batch=B, heads=H, tokens=T, head_dim=D, position=64)
    assert torch.equal(cache[:, :, 64:64 + T], src)

    c16, s16 = (torch.empty(2, 10000, 128, dtype=torch.float16, device="cuda") for _ in range(2))
    kernels.rope_table(c16, s16, theta=1e6, start_position=7)
    ref = np.cos((7 + np.arange(10000, dtype=np.float64))[:, None] * (1e6 ** (-(2 * (np.arange(128) % 64)) / 128)))
    assert np.abs(c16[1].double().cpu().numpy() - ref).max() < 2e-3
    for dt in (torch.float16, torch.float32):
        cd, sd = (torch.empty(2, 10000, 128, dtype=dt, device="cuda") for _ in range(2))
        kernels.rope_table(cd, sd, theta=1e6, start_position=0,
                           start_position_dev=torch.tensor([7], dtype=torch.int64, device="cuda"))
        assert torch.equal(cd.half(), c16) and torch.equal(sd.half(), s16)


def test_asr_encoder_batched_equals_single():
    """forward_batch over three utterances (convolutions over all chunks, linears over all rows, windowed
    attention per utterance) against one forward per utterance: the same rows up to GEMM summation order."""
    import dataclasses

    from torch2vk_b200.asr import AsrEncoderConfig, AsrEncoderRunner, prepare_inputs, random_params

    cfg = dataclasses.replace(AsrEncoderConfig.qwen3_asr_0_6b(), layers=2)
    runner = AsrEncoderRunner(cfg, random_params(cfg, seed=1))
    rng = np.random.default_rng(9)
    clips = [runner.upload(prepare_inputs(rng.standard_normal((cfg.num_mel_bins, 1000)).astype(np.float32), cfg))
             for _ in range(3)]
    batched = runner.forward_batch(clips).float().cpu()
    for b, t in enumerate(clips):
        single = runner.forward(t).float().cpu()
        err = (batched[b] - single).abs().max().item()
        assert err <= 2e-3 * single.abs().max().item(), (b, err)

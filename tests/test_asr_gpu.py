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
                                            (5, 64, 40, True, True)])
def test_linear_q8_0_bias(oracle, m, n, k, bias, gelu):
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

"""The oracle pinned before it is trusted (CPU only).

* golden vectors committed under tests/golden (bytes, decoded floats, matvec);
* gguf-py 0.19.0 (llama.cpp's Python decoders, a third-party package in the
  image): Q4_K / Q6_K / Q8_0 decode bit-exact, Q8_0 quantize bit-exact;
* the reference's GGUF reader (src/torch2vk/checkpoints/gguf.py) parses files
  written by torch2vk_b200.gguf, with the same logical shapes, types and
  physical views (skipped when the reference sources are absent);
* Q4_K_M type topology equals the reference's rules and the layer sets of the
  survey (0.6B / 8B).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
# the reference checkout (read only): T2C_REFERENCE_ROOT, else a `reference` directory beside this
# repository's checkout; tests that need it skip where neither exists
REF_SRC = Path(os.environ.get("T2C_REFERENCE_ROOT", Path(__file__).resolve().parents[2] / "reference")) / "src"
KINDS = ["q8_0", "q4_k", "q6_k"]


@pytest.mark.parametrize("kind", KINDS)
def test_oracle_matches_golden(oracle, kind):
    g = np.load(GOLDEN / f"{kind}.npz")
    packed = oracle.quantize(g["w"], kind)
    assert np.array_equal(packed, g["packed"])
    k = g["w"].shape[1]
    assert np.array_equal(oracle.dequantize(g["packed"], kind, k).view(np.uint32), g["deq"].view(np.uint32))
    assert np.array_equal(oracle.dequantize_np(g["packed"], kind, k).view(np.uint32), g["deq"].view(np.uint32))
    np.testing.assert_allclose(oracle.matvec(g["packed"], kind, g["x"]), g["y"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("kind", KINDS)
def test_oracle_decode_matches_gguf_py(oracle, kind):
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    qt = {"q8_0": Q.Q8_0, "q4_k": Q.Q4_K, "q6_k": Q.Q6_K}[kind]
    rng = np.random.default_rng(21)
    k = 1024
    w = (rng.standard_normal((33, k)) * rng.choice([1e-4, 0.02, 1.0, 30.0], size=(33, 1))).astype(np.float32)
    packed = oracle.quantize(w, kind)
    ref = quants.dequantize(packed, qt)
    got = oracle.dequantize(packed, kind, k)
    assert np.array_equal(ref.view(np.uint32), got.view(np.uint32))
    # arbitrary bytes too (every scale / code pattern), fp16 scales kept finite
    raw = rng.integers(0, 256, size=packed.shape, dtype=np.uint8)
    block = oracle.BLOCK[kind][1]
    view = raw.reshape(-1, block)
    if kind == "q8_0":
        view[:, 0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    elif kind == "q4_k":
        view[:, 0:4] = np.frombuffer(np.array([0.01, 0.002], np.float16).tobytes(), np.uint8)
    else:
        view[:, 208:210] = np.frombuffer(np.float16(0.003).tobytes(), np.uint8)
    assert np.array_equal(quants.dequantize(raw, qt).view(np.uint32), oracle.dequantize(raw, kind, k).view(np.uint32))


def test_oracle_q8_0_quantize_matches_gguf_py(oracle):
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    rng = np.random.default_rng(22)
    w = (rng.standard_normal((17, 512)) * 0.3).astype(np.float32)
    w[0] = 0
    w[1, ::3] = 0.5  # exact .5 multiples exercise the half-away rounding
    assert np.array_equal(quants.quantize(w, Q.Q8_0), oracle.quantize(w, "q8_0"))


def test_oracle_edge_cases(oracle):
    """Empty input, ragged K, and rows with identical values."""
    assert oracle.quantize(np.zeros((0, 256), np.float32), "q4_k").shape == (0, 144)
    with pytest.raises(ValueError):
        oracle.quantize(np.zeros((2, 100), np.float32), "q4_k")
    const = np.full((3, 256), 0.25, np.float32)
    deq = oracle.dequantize(oracle.quantize(const, "q8_0"), "q8_0", 256)
    assert np.all(np.abs(deq - 0.25) < 1e-3)


# ---------------------------------------------------------------- GGUF files
def _write_sample(tmp_path: Path, oracle):
    from torch2vk_b200.gguf import GGMLType, WriteTensor, write_gguf

    rng = np.random.default_rng(5)
    ts = []
    for name, kind, shape in (("blk.q4", "q4_k", (6, 512)), ("blk.q6", "q6_k", (4, 256)), ("blk.q8", "q8_0", (5, 64))):
        w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
        ts.append(WriteTensor(name, oracle.quantize(w, kind), {"q4_k": GGMLType.Q4_K, "q6_k": GGMLType.Q6_K,
                                                              "q8_0": GGMLType.Q8_0}[kind], shape))
    ts.append(WriteTensor("norm", np.arange(7, dtype=np.float32), GGMLType.F32, (7,)))
    ts.append(WriteTensor("embed", np.ones((3, 8), np.float16), GGMLType.F16, (3, 8)))
    path = write_gguf(tmp_path / "model.gguf", ts, extra_u32=(("qwen3.block_count", 2),))
    return path, ts


def test_gguf_roundtrip(tmp_path, oracle):
    from torch2vk_b200.gguf import GGUFFile

    path, ts = _write_sample(tmp_path, oracle)
    with GGUFFile(path) as f:
        assert f.metadata["general.file_type"] == 15 and f.metadata["qwen3.block_count"] == 2
        for t in ts:
            arr = f.array(t.name)
            assert arr.tobytes() == np.ascontiguousarray(t.data).tobytes()
            assert f.tensors[t.name].logical_shape == t.logical_shape
        assert f.array("blk.q4").dtype == np.uint32 and f.array("blk.q4").shape == (6, 72)
        assert f.array("blk.q6").dtype == np.uint16 and f.array("blk.q6").shape == (4, 105)
        assert f.array("blk.q8").dtype == np.uint16 and f.array("blk.q8").shape == (5, 34)


@pytest.mark.skipif(not (REF_SRC / "torch2vk" / "checkpoints" / "gguf.py").is_file(), reason="reference absent")
def test_reference_reader_parses_our_gguf(tmp_path, oracle):
    path, ts = _write_sample(tmp_path, oracle)
    saved = {k: v for k, v in sys.modules.items() if k == "torch2vk" or k.startswith("torch2vk.")}
    for k in saved:
        del sys.modules[k]
    sys.path.insert(0, str(REF_SRC))
    try:
        from torch2vk.checkpoints.gguf import open_gguf_mmap

        with open_gguf_mmap(path) as g:
            assert g.metadata["general.architecture"] == "qwen3"
            for t in ts:
                e = g.tensors[t.name]
                assert tuple(e.logical_shape) == t.logical_shape
                assert int(e.ggml_type) == int(t.ggml_type)
    finally:
        sys.path.remove(str(REF_SRC))
        for k in [k for k in sys.modules if k == "torch2vk" or k.startswith("torch2vk.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_q4_k_m_topology():
    from torch2vk_b200.quantize import GGUFTensorType as T
    from torch2vk_b200.quantize import Q4KMQuantizationConfig, q4_k_m_more_bits_layer_indices

    assert q4_k_m_more_bits_layer_indices(28) == (0, 1, 2, 5, 8, 11, 14, 17, 20, 23, 24, 25, 26, 27)
    eight_b = q4_k_m_more_bits_layer_indices(36)
    assert eight_b[:5] == (0, 1, 2, 3, 6) and eight_b[-6:] == (30, 31, 32, 33, 34, 35) and len(eight_b) == 18
    cfg = Q4KMQuantizationConfig(model_name="m", gguf_arch="qwen3", f16_tensor_names=("model.embed_tokens.weight",),
                                 q6_tensor_names=("lm_head.weight",), q8_tensor_prefixes=("audio.",))
    assert cfg.gguf_type(checkpoint_key="model.embed_tokens.weight", shape=(10, 1024)) is T.F16
    assert cfg.gguf_type(checkpoint_key="lm_head.weight", shape=(10, 1024)) is T.Q6_K
    assert cfg.gguf_type(checkpoint_key="audio.conv.weight", shape=(480, 1, 3, 3)) is T.Q8_0
    assert cfg.gguf_type(checkpoint_key="x.weight", shape=(10, 1024)) is T.Q4_K
    assert cfg.gguf_type(checkpoint_key="x.weight", shape=(10, 96)) is T.Q8_0
    assert cfg.gguf_type(checkpoint_key="x.weight", shape=(10, 100)) is T.F32
    assert cfg.gguf_type(checkpoint_key="x.norm", shape=(1024,)) is T.F32
    assert cfg.gguf_type(checkpoint_key="x.weight", shape=(10, 1024), dtype="int64") is T.F32
    d = cfg.declare_weight(checkpoint_key="audio.conv.weight", dtype="bfloat16", shape=(480, 1, 3, 3))
    assert d.dtype == "uint16" and d.shape == (480, 17)


@pytest.mark.skipif(not (REF_SRC / "torch2vk" / "quantize" / "gguf.py").is_file(), reason="reference absent")
def test_q4_k_m_rules_match_reference_source():
    """The reference's Q4_K_M layer rule, evaluated from its source, for every depth up to 64."""
    import ast

    src = (REF_SRC / "torch2vk" / "quantize" / "gguf.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "q4_k_m_more_bits_layer_indices")
    ns: dict = {}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "ref", "exec"), ns)
    from torch2vk_b200.quantize import q4_k_m_more_bits_layer_indices

    for n in range(1, 65):
        assert ns["q4_k_m_more_bits_layer_indices"](n) == q4_k_m_more_bits_layer_indices(n)


def test_fa_mask_opt_restatement_known_codes():
    """Hand-built masks with known 2-bit codes (fa_mask_opt_f16.py: 1 = all <= -FLT_MAX/2 or outside
    the mask, 2 = all zero, 0 = mixed), words stored [row_block][word]."""
    from oracle import prefill32_ref as ref

    m = np.zeros((20, 1100), np.float16)
    m[:, 64:128] = -np.inf          # block 1: all masked
    m[3, 200] = 1.0                 # block 3 of row block 0: mixed
    m[16:, 256:320] = -np.inf       # block 4 of row block 1 only
    codes = ref.fa_mask_opt(m)
    assert codes.shape == (2, 2)

    def code(rb, blk):
        return (int(codes[rb, blk // 16]) >> (2 * (blk % 16))) & 3

    assert [code(0, b) for b in range(6)] == [2, 1, 2, 0, 2, 2]
    assert [code(1, b) for b in range(6)] == [2, 1, 2, 2, 1, 2]
    assert code(0, 17) == 2 and code(0, 18) == 1            # 1100 columns: block 17 partial, 18 outside
    assert all(code(1, b) == 1 for b in range(18, 32))
    causal = ref.causal_mask(0, 32, 128)
    c = ref.fa_mask_opt(causal)
    assert (int(c[0, 0]) & 3) == 0 and ((int(c[0, 0]) >> 2) & 3) == 1   # diagonal block mixed, next masked

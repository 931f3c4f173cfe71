"""Q4_K_M GGUF export of a safetensors checkpoint (quantize.export_q4_k_m_gguf; the reference's
src/torch2vk/quantize/gguf.py:191-247 entry point).

A tiny Qwen3-shaped checkpoint in two safetensors files (two decoder layers,
norms, an embedding forced to F16, a Q8_0-forced tensor, a tensor whose K is
not a multiple of 256 and one of 32) is exported with the GPU quantizers.
Checked: gguf-py's reader (an independent GGUF implementation, pinned in the
oracle notes) parses the file; every tensor has the type of the config's plan
and its logical shape; every payload equals the CPU oracle's quantization of
the same values (bit for bit); the metadata keys; a second export with the same
plan keeps the file; duplicate names are rejected before anything is written.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, I, V = 256, 512, 320


def _checkpoint(tmp_path):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(0)

    def w(*shape):
        return torch.randn(*shape, generator=g) * 0.02

    a = {"model.embed_tokens.weight": w(V, H), "model.norm.weight": torch.ones(H), "lm_head.weight": w(V, H)}
    b = {}
    for i in range(2):
        p = f"model.layers.{i}."
        b.update({p + "input_layernorm.weight": torch.ones(H), p + "post_attention_layernorm.weight": torch.ones(H),
                  p + "self_attn.q_proj.weight": w(H, H), p + "self_attn.k_proj.weight": w(128, H),
                  p + "self_attn.v_proj.weight": w(128, H), p + "self_attn.o_proj.weight": w(H, H),
                  p + "mlp.gate_proj.weight": w(I, H), p + "mlp.up_proj.weight": w(I, H),
                  p + "mlp.down_proj.weight": w(H, I)})
    b["extra.odd_k.weight"] = w(16, 96)     # K % 256 != 0, K % 32 == 0 -> Q8_0
    b["extra.forced_q8.weight"] = w(8, 256)  # forced Q8_0 by name
    b["extra.tiny.weight"] = w(4, 20)        # K % 32 != 0 -> F32
    d = tmp_path / "ckpt"
    d.mkdir()
    save_file(a, str(d / "model-00001.safetensors"))
    save_file(b, str(d / "model-00002.safetensors"))
    return d, {**a, **b}


def _config():
    from torch2vk_b200.quantize import Q4KMQuantizationConfig, q4_k_m_more_bits_layer_indices

    q6 = tuple(f"model.layers.{i}.{n}.weight" for i in q4_k_m_more_bits_layer_indices(2)
               for n in ("self_attn.v_proj", "mlp.down_proj"))
    return Q4KMQuantizationConfig(model_name="tiny-qwen3", gguf_arch="qwen3",
                                  f16_tensor_names=("model.embed_tokens.weight",),
                                  q6_tensor_names=q6 + ("lm_head.weight",),
                                  q8_tensor_names=("extra.forced_q8.weight",),
                                  extra_uint32_metadata=(("qwen3.block_count", 2),))


def test_export_q4_k_m_gguf(tmp_path, oracle):
    import gguf as gguf_py

    from torch2vk_b200.gguf import GGMLType
    from torch2vk_b200.quantize import export_q4_k_m_gguf

    d, tensors = _checkpoint(tmp_path)
    cfg = _config()
    out = export_q4_k_m_gguf(model_dir=d, output=tmp_path / "out" / "model.gguf", config=cfg)
    reader = gguf_py.GGUFReader(str(out))
    by_name = {t.name: t for t in reader.tensors}
    assert set(by_name) == set(tensors)
    fields = reader.fields
    assert bytes(fields["general.architecture"].parts[-1]).decode() == "qwen3"
    assert int(fields["qwen3.block_count"].parts[-1][0]) == 2
    kinds = {GGMLType.Q4_K: "q4_k", GGMLType.Q6_K: "q6_k", GGMLType.Q8_0: "q8_0"}
    seen = set()
    for name, value in tensors.items():
        arr = value.float().numpy()
        shape = tuple(arr.shape)
        want = cfg.gguf_type(checkpoint_key=name, shape=shape)
        t = by_name[name]
        assert int(t.tensor_type) == int(want), name
        seen.add(want)
        raw = np.asarray(t.data).view(np.uint8).reshape(-1)
        if want in kinds:
            rows = shape[0]
            cols = int(np.prod(shape[1:]))
            if want is GGMLType.Q8_0:
                padded = np.zeros((rows, (cols + 31) // 32 * 32), np.float32)
                padded[:, :cols] = arr.reshape(rows, cols)
                expect = oracle.quantize(padded, "q8_0")
            else:
                expect = oracle.quantize(arr.reshape(rows, cols), kinds[want])
            assert np.array_equal(raw, expect.reshape(-1)), f"{name}: payload differs from the oracle"
        elif want is GGMLType.F16:
            assert np.array_equal(raw.view(np.float16), arr.astype(np.float16).reshape(-1)), name
        else:
            assert np.array_equal(raw.view(np.float32), arr.astype(np.float32).reshape(-1)), name
    assert {GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.Q8_0, GGMLType.F16, GGMLType.F32} <= seen
    # the same plan again: the file is kept (same inode contents, no rewrite)
    stamp = out.stat().st_mtime_ns
    assert export_q4_k_m_gguf(model_dir=d, output=out, config=cfg) == out
    assert out.stat().st_mtime_ns == stamp
    assert not any(p.name.endswith(".partial") for p in out.parent.iterdir())


def test_export_rejects_duplicate_names(tmp_path):
    from safetensors.torch import save_file

    from torch2vk_b200.quantize import export_q4_k_m_gguf

    d = tmp_path / "dup"
    d.mkdir()
    save_file({"a.weight": torch.zeros(4, 256)}, str(d / "x1.safetensors"))
    save_file({"a.weight": torch.zeros(4, 256)}, str(d / "x2.safetensors"))
    out = tmp_path / "dup.gguf"
    with pytest.raises(ValueError, match="twice"):
        export_q4_k_m_gguf(model_dir=d, output=out, config=_config())
    assert not out.exists()

"""A Qwen3 bs1 decode step dispatched through RuntimeSession the way the reference's optimized
model does it (src/models/optimized_qwen3/dispatch/decode_layer.py:36-128 and the greedy head of
src/models/quantized_qwen3/run.py:96-147): per layer RMSNorm, fused Q4_K QKV matvec, q / k RMSNorm +
RoPE transpose, decode attention with the cache write, o_proj + residual, RMSNorm, fused gate / up,
SwiGLU, down_proj + residual; then the final norm, the Q6_K LM-head argmax partials, the two-level
select and the token store.  Weights are seeded random, quantized on the GPU and written to a GGUF
that the session loads, so the step exercises the whole drop-in path (GGUF -> session -> op table
-> libt2c_sm100)."""

from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

from torch2vk_b200 import kernels
from torch2vk_b200.gguf import GGMLType, WriteTensor, write_gguf
from torch2vk_b200.runtime import variants as V
from torch2vk_b200.runtime.logical import LogicalTensor, MemoryClass, TensorLifetime, TensorRole, \
    bind_logical_tensor_alias
from torch2vk_b200.runtime.types import TensorSpec, q4_k_words_layout, q6_k_halfwords_layout

_ROLES = {"act": (TensorRole.ACTIVATION, MemoryClass.FRAME_WORKSPACE, TensorLifetime.FRAME),
          "input": (TensorRole.INPUT, MemoryClass.HOST_INPUT, TensorLifetime.FRAME),
          "state": (TensorRole.STATE, MemoryClass.REQUEST_STATE, TensorLifetime.REQUEST)}


def _t(name: str, dtype: str, shape, role: str = "act") -> LogicalTensor:
    r = _ROLES[role]
    return LogicalTensor(spec=TensorSpec(dtype, tuple(shape)), role=r[0], memory=r[1], lifetime=r[2], name=name)


def _alias(src: LogicalTensor, name: str, shape) -> LogicalTensor:
    a = _t(name, src.spec.dtype, shape)
    bind_logical_tensor_alias(src, a)
    return a


@dataclass
class SessionDecodeModel:
    hidden: int = 1024
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 3072
    layers: int = 28
    vocab: int = 151936
    max_seq: int = 1024
    seed: int = 0
    weights: list = field(default_factory=list)

    def write_gguf(self, directory: Path) -> None:
        """Seeded N(0, 0.02) weights, Q4_K linears and a Q6_K LM head (quantized on the GPU), norms 1."""
        H, NH, NK, D, FF = self.hidden, self.heads, self.kv_heads, self.head_dim, self.intermediate
        gen = torch.Generator(device="cuda").manual_seed(self.seed)
        tensors: list[WriteTensor] = []

        def quant(name, n, k, kind):
            w = torch.randn(n, k, generator=gen, device="cuda") * 0.02
            p = kernels.quantize(w, kind).cpu().numpy().view(np.uint8).reshape(n, -1)
            tensors.append(WriteTensor(name, p, GGMLType.Q4_K if kind == "q4_k" else GGMLType.Q6_K, (n, k)))
            dtype, cols, layout = ("uint32", k // 256 * 36, q4_k_words_layout(logical_k=k)) if kind == "q4_k" else \
                ("uint16", k // 256 * 105, q6_k_halfwords_layout(logical_k=k))
            return LogicalTensor(spec=TensorSpec(dtype, (n, cols)), role=TensorRole.WEIGHT,
                                 memory=MemoryClass.MODEL_WEIGHT, lifetime=TensorLifetime.MODEL, checkpoint_key=name,
                                 layout=layout, name=name)

        def ones(name, n):
            tensors.append(WriteTensor(name, np.ones(n, np.float32), GGMLType.F32, (n,)))
            return LogicalTensor(spec=TensorSpec("float32", (n,)), role=TensorRole.WEIGHT,
                                 memory=MemoryClass.MODEL_WEIGHT, lifetime=TensorLifetime.MODEL, checkpoint_key=name,
                                 name=name)

        self.layer_w = [dict(inn=ones(f"l{i}.in", H), wq=quant(f"l{i}.q", NH * D, H, "q4_k"),
                             wk=quant(f"l{i}.k", NK * D, H, "q4_k"), wv=quant(f"l{i}.v", NK * D, H, "q4_k"),
                             qn=ones(f"l{i}.qn", D), kn=ones(f"l{i}.kn", D), wo=quant(f"l{i}.o", H, NH * D, "q4_k"),
                             post=ones(f"l{i}.post", H), wg=quant(f"l{i}.g", FF, H, "q4_k"),
                             wu=quant(f"l{i}.u", FF, H, "q4_k"), wd=quant(f"l{i}.d", H, FF, "q4_k"))
                        for i in range(self.layers)]
        self.final_norm = ones("final_norm", H)
        self.lm_head = quant("lm_head", self.vocab, H, "q6_k")
        self.weights = [v for lw in self.layer_w for v in lw.values()] + [self.final_norm, self.lm_head]
        write_gguf(Path(directory) / "model.gguf", tensors)
        self._declare()

    def _declare(self) -> None:
        H, NH, NK, D, FF, S = self.hidden, self.heads, self.kv_heads, self.head_dim, self.intermediate, self.max_seq
        G = (self.vocab + 3) // 4
        self.x_in, self.eos = _t("x_in", "float16", (1, 1, H), "input"), _t("eos", "int64", (2,), "input")
        self.k_caches = [_t(f"kc{i}", "float16", (1, S, NK, D), "state") for i in range(self.layers)]
        self.v_caches = [_t(f"vc{i}", "float16", (1, S, NK, D), "state") for i in range(self.layers)]
        self.generated = _t("generated_tokens", "int64", (1, 512), "state")
        self.generated_length, self.stopped = _t("generated_length", "uint32", (1,), "state"), \
            _t("stopped", "uint32", (1,), "state")
        self.cos, self.sin = _t("cos", "float16", (1, 1, D)), _t("sin", "float16", (1, 1, D))
        self.acts = []
        for i in range(self.layers):
            a = dict(hn=_t(f"hn{i}", "float16", (1, 1, H)), q=_t(f"q{i}", "float16", (1, 1, NH * D)),
                     k=_t(f"k{i}", "float16", (1, 1, NK * D)), v=_t(f"v{i}", "float16", (1, 1, NK * D)),
                     qr=_t(f"qr{i}", "float16", (1, NH, 1, D)), kr=_t(f"kr{i}", "float16", (1, NK, 1, D)),
                     att=_t(f"att{i}", "float16", (1, NH, 1, D)), a=_t(f"a{i}", "float16", (1, 1, H)),
                     an=_t(f"an{i}", "float16", (1, 1, H)), g=_t(f"g{i}", "float16", (1, 1, FF)),
                     u=_t(f"u{i}", "float16", (1, 1, FF)), sw=_t(f"sw{i}", "float16", (1, 1, FF)),
                     h=_t(f"h{i + 1}", "float16", (1, 1, H)))
            a["q4"], a["k4"] = _alias(a["q"], f"q4_{i}", (1, 1, NH, D)), _alias(a["k"], f"k4_{i}", (1, 1, NK, D))
            a["v4"] = _alias(a["v"], f"v4_{i}", (1, 1, NK, D))
            a["att3"] = _alias(a["att"], f"att3_{i}", (1, 1, NH * D))
            self.acts.append(a)
        self.fn = _t("fn", "float16", (1, 1, H))
        self.ps, self.pt = _t("ps", "float32", (G,)), _t("pt", "uint32", (G,))
        self.cs, self.ct = _t("cs", "float32", ((G + 1023) // 1024,)), _t("ct", "uint32", ((G + 1023) // 1024,))
        self.next_token, self.done = _t("next_token", "int64", (1, 1)), _t("done", "uint32", (1,))

    def request_state(self) -> dict:
        z = np.zeros((1, self.max_seq, self.kv_heads, self.head_dim), np.float16)
        state = {c: z for c in self.k_caches + self.v_caches}
        state.update({self.generated: np.zeros((1, 512), np.int64),
                      self.generated_length: np.zeros(1, np.uint32), self.stopped: np.zeros(1, np.uint32)})
        return state

    def step(self, rt, position: int, token_index: int) -> None:
        """One decode step's dispatches (286 for 28 layers) inside the caller's frame."""
        V.ROPE_TABLE_F32(rt, cos=self.cos, sin=self.sin, start_position=position, theta=1e6)
        h = self.x_in
        for w, a, kc, vc in zip(self.layer_w, self.acts, self.k_caches, self.v_caches):
            V.RMS_NORM_MUL_F16_F32(rt, x=h, weight=w["inn"], output=a["hn"])
            V.LINEAR_NOBIAS_Q4_K_QKV_MATVEC_F32(rt, x=a["hn"], q_weight=w["wq"], k_weight=w["wk"], v_weight=w["wv"],
                                               q_output=a["q"], k_output=a["k"], v_output=a["v"])
            V.RMS_NORM_ROPE_TRANSPOSE_F16(rt, x=a["q4"], weight=w["qn"], cos=self.cos, sin=self.sin, output=a["qr"])
            V.RMS_NORM_ROPE_TRANSPOSE_F16(rt, x=a["k4"], weight=w["kn"], cos=self.cos, sin=self.sin, output=a["kr"])
            V.SDPA_DECODE_CACHE_WRITE_F32(rt, q=a["qr"], new_k=a["kr"], new_v=a["v4"], k_cache=kc, v_cache=vc,
                                          output=a["att"], cache_position=position)
            V.LINEAR_NOBIAS_Q4_K_MATVEC_ADD_F32(rt, x=a["att3"], weight=w["wo"], residual=h, output=a["a"])
            V.RMS_NORM_MUL_F16_F32(rt, x=a["a"], weight=w["post"], output=a["an"])
            V.LINEAR_NOBIAS_Q4_K_QK_MATVEC_F32(rt, x=a["an"], q_weight=w["wg"], k_weight=w["wu"], q_output=a["g"],
                                              k_output=a["u"])
            V.SWIGLU_F16(rt, gate=a["g"], up=a["u"], output=a["sw"])
            V.LINEAR_NOBIAS_Q4_K_MATVEC_ADD_F32(rt, x=a["sw"], weight=w["wd"], residual=a["a"], output=a["h"])
            h = a["h"]
        V.RMS_NORM_MUL_F16_F32(rt, x=h, weight=self.final_norm, output=self.fn)
        V.LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16(rt, x=self.fn, weight=self.lm_head, partial_scores=self.ps,
                                          partial_tokens=self.pt)
        V.QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32(rt, scores=self.ps, tokens=self.pt, chunk_scores=self.cs,
                                              chunk_tokens=self.ct)
        V.QWEN3_TOKEN_SELECT_REDUCE_F32(rt, partial_scores=self.cs, partial_tokens=self.ct, eos_token_ids=self.eos,
                                        next_token=self.next_token, done=self.done)
        V.QWEN3_TOKEN_STORE_EOS(rt, next_token=self.next_token, done=self.done, generated_tokens=self.generated,
                                generated_length=self.generated_length, stopped=self.stopped, token_index=token_index)

"""CUDA op table: contract class_name -> launcher of libt2c_sm100 kernels.

RuntimeSession.dispatch validates a ShaderVariant call exactly like the
reference dispatcher (src/torch2vk/runtime/dispatcher.py:28-172), then calls
OPS[contract.class_name](rt, variant, buffers, symbols, push) on the
session's CUDA stream.  `buffers` maps field names to the materialized torch
CUDA tensors (declared shape and dtype), `symbols` holds the bound shape
symbols and `push` the resolved push-constant values.  Each entry states the
reference program whose semantics it reproduces.  A class without an entry
raises NotImplementedError at dispatch; nothing falls back to a host path.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from torch2vk_b200 import kernels
from torch2vk_b200.runtime.replay import DynamicPush

OpFn = Callable[..., None]
OPS: dict[str, OpFn] = {}


def op(*class_names: str) -> Callable[[OpFn], OpFn]:
    def deco(fn: OpFn) -> OpFn:
        for name in class_names:
            OPS[name] = fn
        return fn
    return deco


def _positions(rt, batch: int, value: int) -> torch.Tensor:
    return torch.full((batch,), int(value), dtype=torch.int32, device=rt.device)


def _kind_of(weight: torch.Tensor, class_name: str) -> str:
    if "Q6K" in class_name or "Q6_K" in class_name:
        return "q6_k"
    if "Q8_0" in class_name:
        return "q8_0"
    return "q4_k"


# --------------------------------------------------------------------- linear
@op("ExportLinearNobiasQ4KMatvecProgram", "ExportLinearNobiasQ4KProgram",
    "ExportLinearNobiasQ6KMatvecProgram", "ExportLinearNobiasQ6KProgram",
    "ExportLinearNobiasQ8_0MatvecProgram", "ExportLinearNobiasQ8_0Program")
def _linear(rt, variant, b, s, pc):
    """y = x @ deq(W)^T (linear_nobias_{q4_k,q6_k,q8_0}[_matvec]_f32.py)."""
    kind = _kind_of(b["weight"], variant.contract.class_name)
    k = int(s["K"])
    if kind == "q8_0" and b["x"].numel() // k > 8 and k % 256 != 0 and k % 8 == 0:
        # many rows and K not a whole number of 256-value groups: the mma.sync Q8_0 GEMM
        n = b["output"].shape[-1]
        kernels.linear_q8_0_bias(b["x"], b["weight"], None, n, out=b["output"])
        return
    kernels.linear(b["x"], b["weight"], kind, k, out=b["output"])


@op("OptimizedLinearNobiasQ4KMatvecAddProgram", "OptimizedLinearNobiasQ6KMatvecAddProgram")
def _linear_add(rt, variant, b, s, pc):
    """y = residual + x @ deq(W)^T (linear_nobias_q{4,6}_k_matvec_add_f32.py:45-97)."""
    kind = "q6_k" if "Q6K" in variant.contract.class_name else "q4_k"
    kernels.linear(b["x"], b["weight"], kind, s["K"], residual=b["residual"], out=b["output"])


@op("LinearNobiasQ4KQKVMatvecProgram", "LinearNobiasQ4QKQ6VMatvecProgram", "LinearNobiasQ4KQKMatvecProgram")
def _linear_multi(rt, variant, b, s, pc):
    """One x, two or three weight streams (linear_nobias_q4_k_qkv / q4_qk_q6_v / q4_k_qk)."""
    parts = [p for p in ("q", "k", "v") if f"{p}_weight" in b]
    kinds = {"q": "q4_k", "k": "q4_k",
             "v": "q6_k" if variant.contract.class_name == "LinearNobiasQ4QKQ6VMatvecProgram" else "q4_k"}
    kernels.linear_multi(b["x"], [(b[f"{p}_weight"], kinds[p]) for p in parts], s["K"],
                         outs=[b[f"{p}_output"] for p in parts])


# ---------------------------------------------------------------------- norms
@op("ExportRmsNormF32WeightProgram", "OptimizedQwen3RmsNormMulF16F32Program")
def _rms_norm(rt, variant, b, s, pc):
    """fp16(x * rsqrt(mean(x^2) + eps) * w) per row (rms_norm_f32w_f32.py, rms_norm_mul_f16_f32.py:109)."""
    x, out = b["x"], b["output"]
    if x.numel() != out.numel() or b["weight"].numel() != x.shape[-1]:
        raise ValueError(f"{variant.name}: output / weight do not match x {tuple(x.shape)}")
    kernels.rms_norm(x, b["weight"], float(pc.get("eps", 1e-6)), out=out)


@op("OptimizedQwen3RmsNormRopeTransposeF16Program")
def _rms_norm_rope_transpose(rt, variant, b, s, pc):
    """x [B,T,G,D] -> rope(rmsnorm(x)*w) written head-major [B,G,T,D] (rms_norm_rope_transpose_f16.py:22-146)."""
    B, T, G, D = (s[k] for k in ("B", "T", "G", "D"))
    kernels.rms_norm_rope(b["x"], b["weight"], b["cos"], b["sin"], b["output"],
                          out_strides=(G * T * D, T * D, D))


@op("RopeTableF32Program", "RopeTableOutputF32Program")
def _rope_table(rt, variant, b, s, pc):
    """cos/sin [B,T,D] at positions start_position + t, fp16 (runtime/rope_table.py:31-121) or fp32
    (RopeTableOutputF32Program, :124-160)."""
    start = pc["start_position"]
    dev = start.device(torch.int64) if isinstance(start, DynamicPush) else None
    kernels.rope_table(b["cos"], b["sin"], theta=float(pc["theta"]), start_position=0 if dev is not None else int(start),
                       attention_scaling=float(pc.get("attention_scaling", 1.0)), start_position_dev=dev)


# ---------------------------------------------------------------- elementwise
def _as4(t: torch.Tensor) -> torch.Tensor:
    while t.dim() < 4:
        t = t.unsqueeze(0)
    return t


@op("ExportAddF32Program")
def _add(rt, variant, b, s, pc):
    kernels.elementwise4d("add", _as4(b["x"]), _as4(b["y"]), _as4(b["output"]))


@op("ExportMulF32Program", "ExportMulBroadcastProgram")
def _mul(rt, variant, b, s, pc):
    kernels.elementwise4d("mul", _as4(b["x"]), _as4(b["y"]), _as4(b["output"]))


@op("ExportNegF32Program")
def _neg(rt, variant, b, s, pc):
    kernels.elementwise4d("neg", _as4(b["x"]), None, _as4(b["output"]))


@op("ExportSiluF32Program")
def _silu(rt, variant, b, s, pc):
    kernels.elementwise4d("silu", _as4(b["x"]), None, _as4(b["output"]))


@op("OptimizedQwen3SwiGLUF16Program")
def _swiglu(rt, variant, b, s, pc):
    """fp16(silu(gate)) * up (swiglu_f16.py:20-80)."""
    kernels.swiglu(b["gate"], b["up"], out=b["output"])


# ---------------------------------------------------------------------- views
@op("ExportSliceProgram")
def _slice(rt, variant, b, s, pc):
    """out row r = x row r, columns OFFSET .. OFFSET+O3 (slice_f32*.py: IN_STRIDE / OUT_STRIDE / OFFSET)."""
    x, out = b["x"], b["output"]
    in_stride, out_stride, offset = int(pc["IN_STRIDE"]), int(pc["OUT_STRIDE"]), int(pc["OFFSET"])
    rows = out.numel() // out_stride
    if x.numel() != rows * in_stride or offset + out_stride > in_stride:
        raise ValueError(f"{variant.name}: slice of {tuple(x.shape)} to {tuple(out.shape)} at {offset} is not a row slice")
    src = x.reshape(1, 1, rows, in_stride)[..., offset:offset + out_stride]
    kernels.copy4d(src, out.reshape(1, 1, rows, out_stride))


@op("ExportCat2Program")
def _cat2(rt, variant, b, s, pc):
    """Last-dim concatenation (cat_2_f32.py: END0 / STRIDE0 / END1 / STRIDE1)."""
    x0, x1, out = b["x0"], b["x1"], b["output"]
    w0, w1, w = int(pc["STRIDE0"]), int(pc["STRIDE1"]), int(pc["OUT_STRIDE"])
    rows = out.numel() // w
    if w0 + w1 != w or x0.numel() != rows * w0 or x1.numel() != rows * w1:
        raise ValueError(f"{variant.name}: cat of {tuple(x0.shape)} and {tuple(x1.shape)} to {tuple(out.shape)}")
    o = out.reshape(1, 1, rows, w)
    kernels.copy4d(x0.reshape(1, 1, rows, w0), o[..., :w0])
    kernels.copy4d(x1.reshape(1, 1, rows, w1), o[..., w0:])


@op("ExportTransposeProgram")
def _transpose(rt, variant, b, s, pc):
    """out[c0,c1,c2,c3] = x[...] with the variant's dim permutation (transpose_f32_*.py)."""
    from torch2vk_b200.runtime.variants import TRANSPOSE_PERMUTATIONS

    x, out = b["x"], b["output"]
    perm = TRANSPOSE_PERMUTATIONS.get(variant.name)
    if perm is None and variant.name.startswith("transpose_f32"):
        perm = (0, 2, 1, 3)
    if perm is None:
        raise NotImplementedError(f"{variant.name}: unknown transpose permutation")
    if len(perm) != x.dim():
        raise ValueError(f"{variant.name}: rank-{len(perm)} permutation of a rank-{x.dim()} tensor")
    src = x.permute(*perm)
    if tuple(src.shape) != tuple(out.shape):
        raise ValueError(f"{variant.name}: permuted {tuple(src.shape)} != output {tuple(out.shape)}")
    while src.dim() < 4:
        src, out = src.unsqueeze(0), out.unsqueeze(0)
    kernels.copy4d(src, out)


@op("SliceLastTokenF16Program")
def _slice_last(rt, variant, b, s, pc):
    """out[b,0,:] = x[b,S-1,:] (slice_last_token_f16.py)."""
    x, out = b["x"], b["output"]
    kernels.copy4d(x[:, -1:, :].unsqueeze(0), out.unsqueeze(0))


# ---------------------------------------------------------- KV cache / attention
@op("ExportKvCacheWriteF16Program")
def _kv_write(rt, variant, b, s, pc):
    """cache[b,h,pos_t,:] = src[b,h,t,:], pos_t from cache_position[T] or push constant + t
    (kv_cache_write_f16.py:22-92, kv_cache_write_decode_f16.py:23-85)."""
    cache, src = b["cache"], b["src"]
    B, H, S, D, T = (s[k] for k in ("B", "H", "S", "D", "T"))
    pos_t, pos = b.get("cache_position"), pc.get("cache_position", 0)
    if pos_t is None and isinstance(pos, DynamicPush):  # captured replay plan: rows start + t from device memory
        pos.guard(0, S - T + 1)
        pos_t, pos = pos.device(torch.int64, T, ramp=True), 0
    kernels.kv_cache_write(cache, src, cache_strides_bsh=(H * S * D, D, S * D), seq_len=S,
                           src_strides_bth=(H * T * D, D, T * D), batch=B, heads=H, tokens=T, head_dim=D,
                           positions=pos_t, position=int(pos))


@op("OptimizedQwen3TokenMajorKvCacheWriteF16PairProgram", "OptimizedQwen3TokenMajorKvCacheWriteF16TripleProgram")
def _kv_write_token_major(rt, variant, b, s, pc):
    """src [B,T,H,D] written into each token-major cache [B,S?,H,D] at cache_position[t]
    (token_major_kv_cache_write_f16_{pair,triple}.py)."""
    src, pos_t = b["src"], b["cache_position"]
    B, H, D, T = (s[k] for k in ("B", "H", "D", "T"))
    for c in ("a", "b", "c"):
        cache = b.get(f"cache_{c}")
        if cache is None:
            continue
        S = s[f"S{c.upper()}"]
        kernels.kv_cache_write(cache, src, cache_strides_bsh=(S * H * D, H * D, D), seq_len=S,
                               src_strides_bth=(T * H * D, H * D, D), batch=B, heads=H, tokens=T, head_dim=D,
                               positions=pos_t)


@op("ExportSdpaProgram")
def _sdpa(rt, variant, b, s, pc):
    """ExportSdpaProgram: the masked variant (a `mask` field: the ASR encoder's windows) or the causal one."""
    if "mask" in b:
        _sdpa_masked(rt, variant, b, s, pc)
    else:
        _sdpa_causal(rt, variant, b, s, pc)


def _sdpa_causal(rt, variant, b, s, pc):
    """Causal GQA attention, q [B,NH,T,D] over k/v [B,NK,S,D] from position 0 (sdpa_causal_f32.py:22-142)."""
    if "causal" not in variant.name:
        raise NotImplementedError(f"{variant.name}: only causal or masked ExportSdpaProgram variants are served")
    q, k, v, out = b["q"], b["k"], b["v"], b["output"]
    B, NH, T, D = q.shape
    NK, S = k.shape[1], k.shape[2]
    if S < T or tuple(out.shape) != tuple(q.shape) or tuple(v.shape) != tuple(k.shape):
        raise ValueError(f"{variant.name}: q {tuple(q.shape)} k {tuple(k.shape)} out {tuple(out.shape)}")
    kernels.attn_prefill(q, k, v, _positions(rt, B, 0), batch=B, tokens=T, n_heads=NH, n_kv=NK, head_dim=D,
                         layout="head_major", q_layout="head_major", out=out)


def _decode_splits(max_len: int) -> int:
    """Split count of a decode attention over a cache of max_len positions.  Direct frames and captured
    replay plans both take it from the cache length (not the current position), so a replayed step
    combines the same partials in the same order as the direct one: bit-identical results."""
    return max(1, min(64, max_len // 256))


def _decode_at(pc, B: int, S: int, device: torch.device):
    """(write position, attention positions int32 [B], splits) of a decode step at push constant
    cache_position.  The write position is an int, or None past the cache's end (the step writes
    nothing); while a replay plan is captured it is an int64 [1] device slot and the graph serves
    only steps with 0 <= cache_position < S."""
    p = pc["cache_position"]
    if isinstance(p, DynamicPush):
        p.guard(0, S)
        return p.device(torch.int64, 1), p.device(torch.int32, B, clamp_max=S - 1), _decode_splits(S)
    pos = int(p)
    last = min(pos, S - 1)
    positions = torch.full((B,), last, dtype=torch.int32, device=device)
    return (pos if pos < S else None), positions, _decode_splits(S)


def _write_decode_kv(b, wpos, cache_strides, NK: int, D: int, S: int, B: int) -> None:
    if wpos is None:
        return
    dev = isinstance(wpos, torch.Tensor)
    for cache, src, sb in ((b["k_cache"], b["new_k"], D), (b["v_cache"], b["new_v"], NK * D)):
        kernels.kv_cache_write(cache, src, cache_strides_bsh=cache_strides, seq_len=S, src_strides_bth=(NK * D, sb, D),
                               batch=B, heads=NK, tokens=1, head_dim=D, positions=wpos if dev else None,
                               position=0 if dev else wpos)


@op("ExportSdpaDecodeCacheF16Program")
def _sdpa_decode(rt, variant, b, s, pc):
    """One query per head over head-major cache[0..cache_position] (sdpa_decode_cache_f16.py:22-136)."""
    q, k, v, out = b["q"], b["k"], b["v"], b["output"]
    B, NH, NK, S, D = s["B"], s["NH"], s["NK"], s["S"], s["D"]
    if s["T"] != 1:
        raise ValueError(f"{variant.name}: decode attention takes T=1, got {s['T']}")
    p = pc["cache_position"]
    if isinstance(p, DynamicPush):  # captured replay plan: lengths from device memory
        p.guard(0, None)
        positions, splits = p.device(torch.int32, B, clamp_max=S - 1), _decode_splits(S)
    else:
        pos = min(int(p), S - 1)
        positions, splits = _positions(rt, B, pos), _decode_splits(S)
    kernels.attn_decode(q, k, v, positions, batch=B, n_heads=NH, n_kv=NK, head_dim=D, max_len=S,
                        splits=splits, layout="head_major", out=out)


@op("SdpaDecodeCacheWriteF32Program")
def _sdpa_decode_write(rt, variant, b, s, pc):
    """Write new k (head-major) / v (token-major) at cache_position into token-major caches, then
    attend over 0..cache_position (sdpa_decode_cache_write_f32.py:22-171)."""
    q, out = b["q"], b["output"]
    B, NH, NK, S, D = s["B"], s["NH"], s["NK"], s["S"], s["D"]
    if s["T"] != 1:
        raise ValueError(f"{variant.name}: decode attention takes T=1, got {s['T']}")
    wpos, positions, splits = _decode_at(pc, B, S, q.device)
    _write_decode_kv(b, wpos, (S * NK * D, NK * D, D), NK, D, S, B)
    kernels.attn_decode(q, b["k_cache"], b["v_cache"], positions, batch=B, n_heads=NH, n_kv=NK,
                        head_dim=D, max_len=S, splits=splits, layout="token_major", out=out)


# -------------------------------------------------------- embedding / LM head / tokens
@op("ExportEmbeddingQ4_KProgram")
def _embedding_q4k(rt, variant, b, s, pc):
    """out[i,:] = deq(W)[ids[i],:] (embedding_q4_k_f32.py:25-121)."""
    w, ids, out = b["weight"], b["indices"], b["output"]
    kernels.embedding(w, "q4_k", ids, s["H"], w.shape[0], out=out)


@op("LmHeadQ6KArgmaxPartialF16Program")
def _lm_head(rt, variant, b, s, pc):
    """Per-4-row best (score, token) of x @ deq(W)^T (lm_head_q6_k_argmax_partial_f16.py)."""
    G = s["G"]
    if G != (s["N"] + 3) // 4:
        raise ValueError(f"{variant.name}: G={G} but ceil(N/4)={(s['N'] + 3) // 4}")
    kernels.lm_head_argmax(b["x"].reshape(1, s["K"]), b["weight"], "q6_k", s["K"],
                           partial_scores=b["partial_scores"].view(1, G),
                           partial_tokens=b["partial_tokens"].view(torch.int32).view(1, G))


@op("Qwen3TokenSelectReduceChunksF32Program")
def _select_chunks(rt, variant, b, s, pc):
    """Chunks of 1024 partials -> one (score, token) each (qwen3_token_select_reduce_f32.py:21-120)."""
    kernels.token_select_chunks(b["scores"], b["tokens"].view(torch.int32), b["chunk_scores"],
                                b["chunk_tokens"].view(torch.int32))


@op("Qwen3TokenSelectReduceF32Program")
def _select(rt, variant, b, s, pc):
    """Final argmax (lowest token id on ties) and EOS flag (qwen3_token_select_reduce_f32.py:122-241)."""
    G = s["G"]
    kernels.token_select(b["partial_scores"].view(1, G), b["partial_tokens"].view(torch.int32).view(1, G),
                         b["eos_token_ids"], next_token=b["next_token"].view(1),
                         done=b["done"].view(torch.int32).view(1))


@op("Qwen3TokenStoreEosProgram", "Qwen3TokenStoreEosF32Program", "Qwen3TokenStoreProgram",
    "Qwen3AsrTokenStoreEosProgram", "Qwen3AsrTokenStoreProgram")
def _store(rt, variant, b, s, pc):
    """generated_tokens[token_index] = next_token unless stopped; EOS stops (qwen3_token_store.py)."""
    index, dev = pc["token_index"], None
    if isinstance(index, DynamicPush):  # captured replay plan: the index from device memory
        index.guard(-(1 << 31), 1 << 31)
        index, dev = 0, index.device(torch.int32)
    kernels.token_store(b["next_token"].view(1), b["done"].view(torch.int32).view(1), b["generated_tokens"],
                        b["generated_length"].view(torch.int32).view(1), b["stopped"].view(torch.int32).view(1),
                        token_index=int(index), token_index_dev=dev, stop_on_eos=bool(pc.get("stop_on_eos", 1)))


def served_class_names() -> tuple[str, ...]:
    return tuple(sorted(OPS))


# ------------------------------------------------------------ ASR audio encoder
@op("ExportLinearBiasQ8_0WeightF32BiasProgram")
def _linear_bias_q8(rt, variant, b, s, pc):
    """y = x @ deq(W)^T + bias, Q8_0 weights (quantized_qwen3_asr linear_bias_q8_0w_f32b_f32.py:38-92)."""
    kernels.linear_q8_0_bias(b["x"], b["weight"], b["bias"], int(s["N"]), out=b["output"])


@op("ExportConv2dQ8_0WeightF32BiasProgram")
def _conv2d_q8(rt, variant, b, s, pc):
    """NCHW conv2d with Q8_0 weights and fp32 bias (conv2d_q8_0w_f32b_f16.py:36-98)."""
    if pc["kh"] != pc["kw"] or pc["stride_h"] != pc["stride_w"] or pc["pad_h"] != pc["pad_w"]:
        raise NotImplementedError(f"{variant.name}: non-square kernel, stride or padding")
    out = b["output"]
    y = kernels.conv2d_q8_0(b["x"], b["weight"], b["bias"], out.shape[1], kernel=int(pc["kh"]),
                            stride=int(pc["stride_h"]), padding=int(pc["pad_h"]), out=out)
    if tuple(y.shape) != tuple(out.shape):
        raise ValueError(f"{variant.name}: output {tuple(out.shape)} does not match the convolution")


@op("ExportGeluF32Program")
def _gelu(rt, variant, b, s, pc):
    """x * 0.5 * (1 + erf(x / sqrt 2)) (gelu_f32.py; its erf is a 1.5e-7 approximation of the same function)."""
    kernels.gelu(b["x"], out=b["output"])


@op("ExportLayerNormF32WeightF32BiasProgram")
def _layer_norm(rt, variant, b, s, pc):
    """Row LayerNorm, fp32 weight and bias (layer_norm_f32w_f32b_f32.py)."""
    kernels.layer_norm(b["x"], b["weight"], b["bias"], float(pc["eps"]), out=b["output"])


@op("ExportIndexSelectF32Program")
def _index_select(rt, variant, b, s, pc):
    """out[o, :] = x[index[o], :] (index_select_f32_*.py)."""
    kernels.index_rows(b["x"], b["index"], out=b["output"])


def _sdpa_masked(rt, variant, b, s, pc):
    """softmax(q k^T / sqrt(D) + mask) v, non-causal, additive fp16 mask, q [B,NH,T,D] over k / v [B,NK,S,D]
    (sdpa_masked_f32.py:33-90): the ASR encoder's windows (D = 64, as many key heads as query heads) or
    OmniVoice's bidirectional GQA (D = 128, mask [B,1,T,S])."""
    q, k, v, mask, out = b["q"], b["k"], b["v"], b["mask"], b["output"]
    B, NH, T, D = q.shape
    NK = k.shape[1]
    if D == 128:
        m = mask.reshape(mask.shape[0], T, mask.shape[-1]) if mask.dim() == 4 and mask.shape[1] == 1 else mask
        kernels.attn_masked_gqa(q, k, v, m, batch=B, tokens=T, n_heads=NH, n_kv=NK, head_dim=D, layout="head_major",
                                out=out)
        return
    if NK != NH:
        raise NotImplementedError(f"{variant.name}: {NH} query heads over {NK} key heads at D={D}")
    kernels.attn_masked(q, k, v, mask, scale=float(D) ** -0.5, out=out)


@op("OmniVoiceInputEmbedQ8_0Program")
def _omnivoice_input_embed(rt, variant, b, s, pc):
    """Text rows, or the fp32 codebook sum of audio rows, Q8_0 (quantized_omnivoice/custom_shaders.py:17-181)."""
    from torch2vk_b200 import _lib

    ids, amask, out = b["batch_input_ids"], b["batch_audio_mask"], b["hidden_states"]
    B, C, S = ids.shape
    H = out.shape[-1]
    row_bytes = H // 32 * 34
    tw, aw = b["text_weight"], b["audio_weight"]
    tv = tw.numel() * tw.element_size() // row_bytes
    av = aw.numel() * aw.element_size() // row_bytes // C
    if int(pc.get("V", av)) != av:
        raise ValueError(f"{variant.name}: audio table of {av} rows per codebook, push constant V={pc['V']}")
    _lib.lib().call("t2c_omnivoice_input_embed", _lib.ptr(tw), _lib.ptr(aw), _lib.ptr(ids), _lib.ptr(amask),
                    _lib.ptr(out), B, C, S, H, tv, av, _lib.stream_ptr())

# ------------------------------------- fp32-activation prefill (optimized Qwen3, llama.cpp-style)
@op("LlamaMatmulQ4KF32Program", "LlamaMatmulQ6KF32Program")
def _llama_matmul(rt, variant, b, s, pc):
    """output fp32 [X0,X1,N] = x fp32 [X0,X1,K] @ deq(W)^T (llama_matmul_q{4,6}_k_f32.py; the reference
    multiplies fp16 operands with fp16 accumulation, the tensor-core GEMM here accumulates in fp32)."""
    kind = "q6_k" if "Q6K" in variant.contract.class_name else "q4_k"
    kernels.linear_f32(b["x"], b["weight"], kind, s["K"], out=b["output"])


@op("OptimizedQwen3RmsNormMulF32Program")
def _rms_norm_f32(rt, variant, b, s, pc):
    """x * rsqrt(mean(x^2) + 1e-6) * w, fp32 (rms_norm_mul_f32.py)."""
    kernels.rms_norm_f32(b["x"], b["weight"], 1e-6, out=b["output"])


@op("OptimizedQwen3RmsNormRopeTokenF32Program", "OptimizedQwen3RmsNormRopeTokenF32ToF16Program")
def _rms_norm_rope_token(rt, variant, b, s, pc):
    """Per (b, t, head) row: RMSNorm (1e-6) * w then rotate-half RoPE from the fp16 cos / sin tables
    (rms_norm_rope_token_f32.py:22; the _to_f16 variant stores fp16)."""
    kernels.rms_norm_rope_f32(b["x"], b["weight"], b["cos"], b["sin"], b["output"], eps=1e-6)


@op("AddF32PrefillProgram")
def _add_f32(rt, variant, b, s, pc):
    """x + y in fp32 (add_f32_prefill.py)."""
    kernels.add_f32(b["x"], b["y"], out=b["output"])


@op("SwigluF32Program")
def _swiglu_f32(rt, variant, b, s, pc):
    """gate / (1 + exp(-gate)) * up in fp32 (swiglu_f32.py)."""
    kernels.swiglu_f32(b["gate"], b["up"], out=b["output"])


@op("SliceLastTokenF32ToF16Program")
def _slice_last_f32(rt, variant, b, s, pc):
    """output[b,0,:] = fp16(x[b,S-1,:]) (slice_last_token_f32_to_f16.py)."""
    kernels.slice_last_f32_to_f16(b["x"], b["output"])


@op("OptimizedQwen3TokenMajorValueCacheWriteF32ToF16PairProgram",
    "OptimizedQwen3TokenMajorValueCacheWriteF32ToF16TripleProgram")
def _value_cache_write_f32(rt, variant, b, s, pc):
    """fp16(src [B,T,H,D]) into each token-major cache at cache_position[t]; a cache too short for
    the row is skipped (token_major_value_cache_write_f32_to_f16_{pair,triple}.py)."""
    caches = [b[f"cache_{c}"] for c in ("a", "b", "c") if f"cache_{c}" in b]
    kernels.value_cache_write_f32(b["src"], b["cache_position"], caches)


@op("OptimizedQwen3FaMaskOptF16Program")
def _fa_mask_opt(rt, variant, b, s, pc):
    """2-bit all-masked / all-zero codes per 16 x 64 block of the mask (fa_mask_opt_f16.py), stored as
    the shader does: word w of row block r at r * W + w."""
    W, R = s["W"], s["R"]
    if W != (s["S"] + 1023) // 1024 or R != (s["T"] + 15) // 16:
        raise ValueError(f"{variant.name}: output ({W}, {R}) does not cover mask ({s['T']}, {s['S']})")
    kernels.fa_mask_opt(b["mask"], b["output"])


@op("LlamaFlashAttnF32F16F16Program")
def _llama_flash_attn(rt, variant, b, s, pc):
    """softmax(q k^T * scale + mask) v with fp32 q / output [B,T,NH,D] and fp16 token-major caches
    [B,S,NK,D] (llama_flash_attn_f32_f16_f16.py:35-158; no attention sinks: bit 24 of
    mask_n_head_log2 is clear in every reference call)."""
    if int(pc.get("mask_n_head_log2", 0)) & (1 << 24):
        raise NotImplementedError(f"{variant.name}: attention sinks are not served")
    if float(pc.get("logit_softcap", 0.0)) != 0.0 or float(pc.get("max_bias", 0.0)) != 0.0:
        raise NotImplementedError(f"{variant.name}: logit softcap / ALiBi bias are not served")
    kernels.attn_prefill_masked_f32(b["q"], b["k"], b["v"], b["mask"], b.get("mask_opt"), b["output"],
                                    scale=float(pc["scale"]))


@op("OptimizedQwen3EmbeddingQ4KActF32Program")
def _embedding_q4k_f32(rt, variant, b, s, pc):
    """output fp32 [I0,I1,H] = dequantized Q4_K rows (embedding_q4_k_act_f32.py)."""
    w = b["weight"]
    kernels.embedding_f32(w, "q4_k", b["indices"], s["H"], w.shape[0], out=b["output"])


# ------------------------------------------------------------- GGUF quantizers
@op("GGUFQuantizeQ4KF32Program", "GGUFQuantizeQ6KF32Program", "GGUFQuantizeQ8_0F32Program")
def _gguf_quantize(rt, variant, b, s, pc):
    """fp32 [R, K] -> packed blocks, bit-exact with the reference quantizers (quantize/vulkan.py:91-637)."""
    name = variant.contract.class_name
    kind = "q4_k" if "Q4K" in name else "q6_k" if "Q6K" in name else "q8_0"
    kernels.quantize(b["x"], kind, out=b["output"])


# ------------------------------------------------------ ASR text decoder
@op("ExportEmbeddingQ8_0Program")
def _embedding_q8_0(rt, variant, b, s, pc):
    """output fp16 [I0,I1,H] = d * q of Q8_0 rows (quantized_qwen3_asr embedding_q8_0_f32.py)."""
    w = b["weight"]
    kernels.embedding_q8_0(w, b["indices"], s["H"], w.shape[0], out=b["output"])


@op("ExportIndexCopyF32Program")
def _index_copy(rt, variant, b, s, pc):
    """cache[b, index[s], :] = src[b, s, :] (index_copy_f32_*.py: the audio-token injection)."""
    kernels.index_copy_rows(b["cache"], b["index"], b["src"])


# ------------------------------------------------ optimized Qwen3-ASR text decoder
@op("LinearNobiasQ4KPairProgram", "LinearNobiasQ4KTripleProgram")
def _linear_pair_triple(rt, variant, b, s, pc):
    """Two / three Q4_K weights sharing x, one fused launch (optimized_qwen3_asr
    linear_nobias_q4_k_{pair,triple}_f32.py; the reference accumulates in fp16, here fp32)."""
    parts = [i for i in range(3) if f"weight{i}" in b]
    kernels.linear_multi(b["x"], [(b[f"weight{i}"], "q4_k") for i in parts], s["K"],
                         outs=[b[f"output{i}"] for i in parts])


@op("OptimizedQwen3SdpaCausalCacheWriteProgram")
def _sdpa_causal_cache_write(rt, variant, b, s, pc):
    """Writes k (head-major) / v (token-major) rows into head-major caches at cache_position[t]
    (a row past S skipped), then causal attention of the chunk's queries over the chunk's own keys
    (optimized_qwen3_asr sdpa_causal_cache_write_f16.py)."""
    q, k, v, out = b["q"], b["k"], b["v"], b["output"]
    B, NH, NK, T, S, D = (s[x] for x in ("B", "NH", "NK", "T", "S", "D"))
    if T > S:
        raise NotImplementedError(f"{variant.name}: T={T} above the cache length S={S}")
    pos = b["cache_position"]
    cs = (NK * S * D, D, S * D)
    kernels.kv_cache_write(b["k_cache"], k, cache_strides_bsh=cs, seq_len=S, src_strides_bth=(NK * T * D, D, T * D),
                           batch=B, heads=NK, tokens=T, head_dim=D, positions=pos)
    kernels.kv_cache_write(b["v_cache"], v, cache_strides_bsh=cs, seq_len=S, src_strides_bth=(T * NK * D, NK * D, D),
                           batch=B, heads=NK, tokens=T, head_dim=D, positions=pos)
    vh = torch.empty(B, NK, T, D, dtype=torch.float16, device=v.device)
    kernels.copy4d(v.permute(0, 2, 1, 3), vh)
    kernels.attn_prefill(q, k, vh, torch.zeros(B, dtype=torch.int32, device=q.device), batch=B, tokens=T, n_heads=NH, n_kv=NK, head_dim=D, layout="head_major",
                         q_layout="head_major", out=out)


@op("SdpaDecodeCacheWriteF16Program")
def _sdpa_decode_write_f16(rt, variant, b, s, pc):
    """Writes new k (head-major) / v (token-major) at cache_position into head-major caches, then one
    query per head over 0..min(cache_position, S - 1) (optimized_qwen3_asr sdpa_decode_cache_write_f16.py)."""
    q, out = b["q"], b["output"]
    B, NH, NK, S, D = s["B"], s["NH"], s["NK"], s["S"], s["D"]
    if s["T"] != 1:
        raise ValueError(f"{variant.name}: decode attention takes T=1, got {s['T']}")
    wpos, positions, splits = _decode_at(pc, B, S, q.device)
    _write_decode_kv(b, wpos, (NK * S * D, D, S * D), NK, D, S, B)
    kernels.attn_decode(q, b["k_cache"], b["v_cache"], positions, batch=B, n_heads=NH, n_kv=NK, head_dim=D,
                        max_len=S, splits=splits, layout="head_major", out=out)


# unfused RMSNorm chain of the exported text norm (optimized_qwen3_asr shaders)
@op("ExportPowScalarF32Program")
def _pow_scalar(rt, variant, b, s, pc):
    """x * x (pow_scalar_f32.py: exponent 2, fp16 in, fp32 out)."""
    if variant.source not in ("cuda", "") and "v * v" not in variant.source:
        raise NotImplementedError(f"{variant.name}: only the exponent-2 program is served")
    kernels.ew_misc("pow2", b["x"], b["output"])


@op("ExportRsqrtF32Program")
def _rsqrt(rt, variant, b, s, pc):
    """1 / sqrt(x) in fp32 (rsqrt_f32.py)."""
    kernels.ew_misc("rsqrt", b["x"], b["output"])


@op("ExportAddScalarProgram")
def _add_scalar(rt, variant, b, s, pc):
    """x + scalar (add_scalar.py; the scalar is a push constant, 1e-6 for the norm's eps)."""
    kernels.ew_misc("add_scalar", b["x"], b["output"], scalar=float(pc["scalar"]))


@op("ExportMeanDimProgram")
def _mean_dim(rt, variant, b, s, pc):
    """Mean over the last dim, fp32 (mean_dim_f32.py)."""
    kernels.row_mean_f32(b["x"], b["output"])


@op("ExportMulBroadcastLastProgram")
def _mul_broadcast_last(rt, variant, b, s, pc):
    """fp16(x[t, h] * y[t]) (mul_broadcast_last.py: y [1, T, 1] fp32)."""
    kernels.ew_misc("mul_row", b["x"], b["output"], b["y"], H=int(pc["H"]))


@op("ExportMulLeftBroadcastF32XProgram")
def _mul_left_broadcast(rt, variant, b, s, pc):
    """fp16(y[t, h] * x[h]) (mul_left_broadcast_f32x_f32.py: x [H] fp32 weight, y fp16)."""
    kernels.ew_misc("mul_col", b["y"], b["output"], b["x"], H=int(pc["H"]))

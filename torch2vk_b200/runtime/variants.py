"""Hot-path op declarations for the CUDA backend, under the reference's variant names.

Each constant mirrors one reference ShaderVariant of the quantized / optimized
Qwen3 decode path: same variant name, contract class_name, field names, io
kinds, dtypes, symbolic shapes, weight layouts and push-constant names (the
interface a generated dispatch module calls with `VARIANT(rt, **fields)`).
There is no GLSL here: RuntimeSession.dispatch resolves class_name in
torch2vk_b200.runtime.optable and launches the sm_100a kernels.

Reference declarations mirrored (src/models/...):
  quantized_qwen3/shaders/linear_nobias_{q4_k,q6_k,q8_0}{,_matvec}_f32.py,
  rms_norm_f32w_f32.py, add_f32.py, mul_f32.py, mul_broadcast.py, neg_f32.py,
  silu_f32.py, slice_f32.py, cat_2_f32.py, transpose_f32_*.py,
  kv_cache_write_f16.py, kv_cache_write_decode_f16.py, sdpa_causal_f32.py,
  sdpa_decode_cache_f16.py, embedding_q4_k_f32.py,
  lm_head_q6_k_argmax_partial_f16.py, qwen3_token_select_reduce*_f32.py,
  qwen3_token_store_eos.py;
  optimized_qwen3/shaders/linear_nobias_q4_k_{qkv,qk}_matvec_f32.py,
  linear_nobias_q4_qk_q6_v_matvec_f32.py, linear_nobias_q{4,6}_k_matvec_add_f32.py,
  rms_norm_mul_f16_f32.py, rms_norm_rope_transpose_f16.py, swiglu_f16.py,
  token_major_kv_cache_write_f16_{pair,triple}.py, sdpa_decode_cache_write_f32.py,
  slice_last_token_f16.py; src/torch2vk/runtime/rope_table.py:31-121.
"""

from __future__ import annotations

from torch2vk_b200.runtime.shader import (
    IOKind,
    PushConstantFieldSpec,
    PushConstantInput,
    PushConstantSpec,
    PushConstantType,
    ShaderContract,
    ShaderVariant,
    TensorContract,
    TensorFieldSpec,
    add,
    ceil_div,
    mul,
)
from torch2vk_b200.runtime.types import q4_k_words_layout, q6_k_halfwords_layout, q8_0_halfwords_layout

U32, I32, F32 = PushConstantType.UINT32, PushConstantType.INT32, PushConstantType.FLOAT32
IN, OUT, INOUT = IOKind.INPUT, IOKind.OUTPUT, IOKind.INOUT


def _t(name, io, dtype, shape, layout=None, role=None):
    role = role or {IN: "input", OUT: "output", INOUT: "state"}[io]
    c = TensorContract(dtype=dtype, shape=tuple(shape)) if layout is None else TensorContract(
        dtype=dtype, shape=tuple(shape), layout=layout)
    return TensorFieldSpec(name=name, io_kind=io, role=role, contract=c)


def _pcs(*items):
    """items: (name, type, value[, dynamic]); offsets packed in order like std430 scalars."""
    fields, off = [], 0
    for it in items:
        name, ty, value = it[:3]
        dyn = it[3] if len(it) > 3 else False
        fields.append(PushConstantFieldSpec(name, ty, off, value, dynamic=dyn))
        off += 8 if ty is PushConstantType.UINT64 else 4
    return PushConstantSpec(size=off, fields=tuple(fields))


def _named_roles(fields):
    """Contracts of the token-selection family use the field name as the field role."""
    return [TensorFieldSpec(name=f.name, io_kind=f.io_kind, role=f.name, contract=f.contract) for f in fields]


def _v(name, family, class_name, fields, dispatch, pcs=None, source="cuda"):
    return ShaderVariant(name=name, family=family, source=source, contract=ShaderContract(
        class_name=class_name, shader_name=name, fields=tuple(fields), dispatch=dispatch, push_constants=pcs))


M_X = mul("X0", "X1")

# ------------------------------------------------------------------ quantized linear
_WEIGHTS = {
    "q4_k": ("uint32", lambda k: mul(ceil_div(k, 256), 36), lambda k: q4_k_words_layout(logical_k=k)),
    "q6_k": ("uint16", lambda k: mul(ceil_div(k, 256), 105), lambda k: q6_k_halfwords_layout(logical_k=k)),
    "q8_0": ("uint16", lambda k: mul(ceil_div(k, 32), 17), lambda k: q8_0_halfwords_layout(logical_k=k)),
}


def _wfield(name: str, kind: str, rows: str, k: str = "K") -> TensorFieldSpec:
    dtype, words, layout = _WEIGHTS[kind]
    return _t(name, IN, dtype, (rows, words(k)), layout(k), role="weight")


def _linear(kind: str, matvec: bool) -> ShaderVariant:
    name = f"linear_nobias_{kind}{'_matvec' if matvec else ''}_f32"
    cls = {"q4_k": "Q4K", "q6_k": "Q6K", "q8_0": "Q8_0"}[kind]
    class_name = f"ExportLinearNobias{cls}{'Matvec' if matvec else ''}Program"
    if matvec:
        dispatch = (ceil_div("N", 2), M_X, 1)
    elif kind == "q8_0":
        dispatch = (ceil_div(M_X, 32), ceil_div("N", 16), 1)
    else:
        dispatch = (ceil_div("N", 64), ceil_div(M_X, 64), 1)
    return _v(name, "export", class_name,
              [_t("x", IN, "float16", ("X0", "X1", "K")), _wfield("weight", kind, "N"),
               _t("output", OUT, "float16", ("X0", "X1", "N"))],
              dispatch, _pcs(("M", U32, M_X), ("K", U32, "K"), ("N", U32, "N")))


LINEAR_NOBIAS_Q4_K_MATVEC_F32 = _linear("q4_k", True)
LINEAR_NOBIAS_Q4_K_F32 = _linear("q4_k", False)
LINEAR_NOBIAS_Q6_K_MATVEC_F32 = _linear("q6_k", True)
LINEAR_NOBIAS_Q6_K_F32 = _linear("q6_k", False)
LINEAR_NOBIAS_Q8_0_MATVEC_F32 = _linear("q8_0", True)
LINEAR_NOBIAS_Q8_0_F32 = _linear("q8_0", False)


def _matvec_add(kind: str) -> ShaderVariant:
    cls = {"q4_k": "Q4K", "q6_k": "Q6K"}[kind]
    return _v(f"linear_nobias_{kind}_matvec_add_f32", "optimized_qwen3", f"OptimizedLinearNobias{cls}MatvecAddProgram",
              [_t("x", IN, "float16", ("X0", "X1", "K")), _wfield("weight", kind, "N"),
               _t("residual", IN, "float16", ("X0", "X1", "N")), _t("output", OUT, "float16", ("X0", "X1", "N"))],
              (ceil_div("N", 2), M_X, 1), _pcs(("M", U32, M_X), ("K", U32, "K"), ("N", U32, "N")))


LINEAR_NOBIAS_Q4_K_MATVEC_ADD_F32 = _matvec_add("q4_k")
LINEAR_NOBIAS_Q6_K_MATVEC_ADD_F32 = _matvec_add("q6_k")


def _multi(name: str, class_name: str, parts: list[tuple[str, str, str]]) -> ShaderVariant:
    """parts: (prefix, kind, rows symbol), e.g. ("q", "q4_k", "NQ")."""
    fields = [_t("x", IN, "float16", ("X0", "X1", "K"))]
    fields += [_wfield(f"{p}_weight", kind, rows) for p, kind, rows in parts]
    fields += [_t(f"{p}_output", OUT, "float16", ("X0", "X1", rows)) for p, _, rows in parts]
    total = parts[0][2]
    for _, _, rows in parts[1:]:
        total = add(total, rows)
    pcs = [("M", U32, M_X), ("K", U32, "K")] + [(rows, U32, rows) for _, _, rows in parts]
    return _v(name, "optimized_qwen3", class_name, fields, (ceil_div(total, 2), M_X, 1), _pcs(*pcs))


LINEAR_NOBIAS_Q4_K_QKV_MATVEC_F32 = _multi("linear_nobias_q4_k_qkv_matvec_f32", "LinearNobiasQ4KQKVMatvecProgram",
                                           [("q", "q4_k", "NQ"), ("k", "q4_k", "NK"), ("v", "q4_k", "NV")])
LINEAR_NOBIAS_Q4_QK_Q6_V_MATVEC_F32 = _multi("linear_nobias_q4_qk_q6_v_matvec_f32",
                                             "LinearNobiasQ4QKQ6VMatvecProgram",
                                             [("q", "q4_k", "NQ"), ("k", "q4_k", "NK"), ("v", "q6_k", "NV")])
LINEAR_NOBIAS_Q4_K_QK_MATVEC_F32 = _multi("linear_nobias_q4_k_qk_matvec_f32", "LinearNobiasQ4KQKMatvecProgram",
                                          [("q", "q4_k", "NQ"), ("k", "q4_k", "NK")])

# ------------------------------------------------------------------ norms / rope
RMS_NORM_F32W_F32 = _v(
    "rms_norm_f32w_f32", "export", "ExportRmsNormF32WeightProgram",
    [_t("x", IN, "float16", ("I0", "I1", "I2")), _t("weight", IN, "float32", ("C",), role="weight"),
     _t("output", OUT, "float16", ("O0", "O1", "O2"))],
    (mul("I0", "I1"), 1, 1), _pcs(("ROWS", U32, mul("I0", "I1")), ("COLS", U32, "I2"), ("eps", F32, 1e-6)))
RMS_NORM_F32W_F32_2 = _v(
    "rms_norm_f32w_f32_2", "export", "ExportRmsNormF32WeightProgram",
    [_t("x", IN, "float16", ("I0", "I1", "I2", "I3")), _t("weight", IN, "float32", ("C",), role="weight"),
     _t("output", OUT, "float16", ("O0", "O1", "O2", "O3"))],
    (mul(mul("I0", "I1"), "I2"), 1, 1),
    _pcs(("ROWS", U32, mul(mul("I0", "I1"), "I2")), ("COLS", U32, "I3"), ("eps", F32, 1e-6)))
RMS_NORM_MUL_F16_F32 = _v(
    "rms_norm_mul_f16_f32", "optimized_qwen3", "OptimizedQwen3RmsNormMulF16F32Program",
    [_t("x", IN, "float16", ("B", "T", "H")), _t("weight", IN, "float32", ("H",), role="weight"),
     _t("output", OUT, "float16", ("B", "T", "H"))],
    (mul("B", "T"), 1, 1), _pcs(("ROWS", U32, mul("B", "T")), ("H", U32, "H")))
RMS_NORM_ROPE_TRANSPOSE_F16 = _v(
    "rms_norm_rope_transpose_f16", "optimized_qwen3", "OptimizedQwen3RmsNormRopeTransposeF16Program",
    [_t("x", IN, "float16", ("B", "T", "G", "D")), _t("weight", IN, "float32", ("D",), role="weight"),
     _t("cos", IN, "float16", ("B", "T", "D")), _t("sin", IN, "float16", ("B", "T", "D")),
     _t("output", OUT, "float16", ("B", "G", "T", "D"))],
    (mul(mul("B", "T"), "G"), 1, 1),
    _pcs(("ROWS", U32, mul(mul("B", "T"), "G")), ("T", U32, "T"), ("G", U32, "G"), ("D", U32, "D")))
ROPE_TABLE_F32 = _v(
    "rope_table_f32", "torch2vk.rope", "RopeTableF32Program",
    [_t("cos", OUT, "float16", ("B", "T", "D")), _t("sin", OUT, "float16", ("B", "T", "D"))],
    (ceil_div(mul(mul("B", "T"), "D"), 256), 1, 1),
    _pcs(("B", U32, "B"), ("T", U32, "T"), ("D", U32, "D"), ("attention_scaling", F32, 1.0),
         ("theta", F32, PushConstantInput("theta")), ("start_position", U32, PushConstantInput("start_position"))))

# ------------------------------------------------------------------ elementwise
_N3 = mul("T", "H")
_N4 = mul(mul("T", "H"), "D")


def _ew(name: str, class_name: str, rank4: bool, binary: bool) -> ShaderVariant:
    shape = (1, "T", "H", "D") if rank4 else (1, "T", "H")
    n = _N4 if rank4 else _N3
    fields = [_t("x", IN, "float16", shape)] + ([_t("y", IN, "float16", shape)] if binary else [])
    fields.append(_t("output", OUT, "float16", shape))
    return _v(name, "export", class_name, fields, (ceil_div(n, 256), 1, 1), _pcs(("N", U32, n)))


ADD_F32 = _ew("add_f32", "ExportAddF32Program", True, True)
ADD_F32_18 = _ew("add_f32_18", "ExportAddF32Program", False, True)
MUL_F32 = _ew("mul_f32", "ExportMulF32Program", False, True)
NEG_F32 = _ew("neg_f32", "ExportNegF32Program", True, False)
SILU_F32 = _ew("silu_f32", "ExportSiluF32Program", False, False)


def _mul_broadcast(name: str, x_shape, y_shape) -> ShaderVariant:
    return _v(name, "export", "ExportMulBroadcastProgram",
              [_t("x", IN, "float16", x_shape), _t("y", IN, "float16", y_shape),
               _t("output", OUT, "float16", (1, "T", "H", "D"))],
              (ceil_div(_N4, 256), 1, 1),
              _pcs(("N", U32, _N4), ("D0", U32, 1), ("D1", U32, "T"), ("D2", U32, "H"), ("D3", U32, "D")))


MUL_BROADCAST = _mul_broadcast("mul_broadcast", (1, "T", "H", "D"), (1, 1, "H", "D"))
DECODE_LAYER_MUL_BROADCAST = _mul_broadcast("decode_layer_mul_broadcast", (1, "T", 1, "D"), (1, 1, 1, "D"))
SWIGLU_F16 = _v(
    "swiglu_f16", "optimized_qwen3", "OptimizedQwen3SwiGLUF16Program",
    [_t("gate", IN, "float16", ("B", "T", "H")), _t("up", IN, "float16", ("B", "T", "H")),
     _t("output", OUT, "float16", ("B", "T", "H"))],
    (ceil_div(mul(mul("B", "T"), "H"), 256), 1, 1), _pcs(("N", U32, mul(mul("B", "T"), "H"))))

# ------------------------------------------------------------------ views / copies
_O4 = ("O0", "O1", "O2", "O3")
_NOUT = mul(mul(mul("O0", "O1"), "O2"), "O3")


def _slice(name: str, offset) -> ShaderVariant:
    return _v(name, "export", "ExportSliceProgram",
              [_t("x", IN, "float16", ("I0", "I1", "I2", "I3")), _t("output", OUT, "float16", _O4)],
              (ceil_div(_NOUT, 256), 1, 1),
              _pcs(("N_OUT", U32, _NOUT), ("IN_STRIDE", U32, mul("I3", 1)), ("OUT_STRIDE", U32, mul("O3", 1)),
                   ("OFFSET", U32, offset)))


SLICE_F32 = _slice("slice_f32", 0)
SLICE_F32_10 = _slice("slice_f32_10", mul(64, 1))
CAT_2_F32 = _v(
    "cat_2_f32", "export", "ExportCat2Program",
    [_t("x0", IN, "float16", ("I0_0", "I0_1", "I0_2", "I0_3")), _t("x1", IN, "float16", ("I1_0", "I1_1", "I1_2", "I1_3")),
     _t("output", OUT, "float16", _O4)],
    (ceil_div(_NOUT, 256), 1, 1),
    _pcs(("N_OUT", U32, _NOUT), ("OUT_STRIDE", U32, mul("O3", 1)), ("END0", U32, mul("I0_3", 1)),
         ("STRIDE0", U32, mul("I0_3", 1)), ("END1", U32, add(mul("I0_3", 1), mul("I1_3", 1))),
         ("STRIDE1", U32, mul("I1_3", 1))))
TRANSPOSE_F32 = _v(
    "transpose_f32", "export", "ExportTransposeProgram",
    [_t("x", IN, "float16", ("I0", "I1", "I2", "I3")), _t("output", OUT, "float16", _O4)],
    (ceil_div(_NOUT, 256), 1, 1),
    _pcs(("N", U32, _NOUT), *[(s, U32, s) for s in ("O0", "O1", "O2", "O3", "I0", "I1", "I2", "I3")]))
SLICE_LAST_TOKEN_F16 = _v(
    "slice_last_token_f16", "optimized_qwen3", "SliceLastTokenF16Program",
    [_t("x", IN, "float16", ("B", "S", "H")), _t("output", OUT, "float16", ("B", 1, "H"))],
    (ceil_div("H", 256), "B", 1), _pcs(("B", U32, "B"), ("S", U32, "S"), ("H", U32, "H")))

# ------------------------------------------------------------------ KV cache / attention
KV_CACHE_WRITE_F16 = _v(
    "kv_cache_write_f16", "export", "ExportKvCacheWriteF16Program",
    [_t("cache", INOUT, "float16", ("B", "H", "S", "D")), _t("cache_position", IN, "int64", ("T",), role="cache_position"),
     _t("src", IN, "float16", ("B", "H", "T", "D"))],
    (ceil_div(mul(mul(mul("B", "H"), "T"), "D"), 256), 1, 1),
    _pcs(("B", U32, "B"), ("H", U32, "H"), ("S", U32, "S"), ("D", U32, "D"), ("T", U32, "T")))
KV_CACHE_WRITE_DECODE_F16 = _v(
    "kv_cache_write_decode_f16", "export", "ExportKvCacheWriteF16Program",
    [_t("cache", INOUT, "float16", ("B", "H", "S", "D")), _t("src", IN, "float16", ("B", "H", "T", "D"))],
    (ceil_div(mul(mul(mul("B", "H"), "T"), "D"), 256), 1, 1),
    _pcs(("B", U32, "B"), ("H", U32, "H"), ("S", U32, "S"), ("D", U32, "D"), ("T", U32, "T"),
         ("cache_position", U32, PushConstantInput("cache_position"))))


def _token_major_write(name: str, class_name: str, caches: str, src_dtype: str) -> ShaderVariant:
    fields = [_t(f"cache_{c}", INOUT, "float16", ("B", f"S{c.upper()}", "H", "D")) for c in caches]
    fields += [_t("cache_position", IN, "int64", ("T",), role="cache_position"),
               _t("src", IN, src_dtype, ("B", "T", "H", "D"))]
    pcs = [("B", U32, "B")] + [(f"S{c.upper()}", U32, f"S{c.upper()}") for c in caches]
    pcs += [("H", U32, "H"), ("D", U32, "D"), ("T", U32, "T")]
    return _v(name, "optimized_qwen3", class_name, fields,
              (ceil_div(mul(mul(mul("B", "T"), "H"), "D"), 256), 1, 1), _pcs(*pcs))


TOKEN_MAJOR_KV_CACHE_WRITE_F16_PAIR = _token_major_write(
    "token_major_kv_cache_write_f16_pair", "OptimizedQwen3TokenMajorKvCacheWriteF16PairProgram", "ab", "float16")
TOKEN_MAJOR_KV_CACHE_WRITE_F16_TRIPLE = _token_major_write(
    "token_major_kv_cache_write_f16_triple", "OptimizedQwen3TokenMajorKvCacheWriteF16TripleProgram", "abc", "float16")
SDPA_CAUSAL_F32 = _v(
    "sdpa_causal_f32", "export", "ExportSdpaProgram",
    [_t("q", IN, "float16", ("Q0", "Q1", "Q2", "Q3")), _t("k", IN, "float16", ("K0", "K1", "K2", "K3")),
     _t("v", IN, "float16", ("V0", "V1", "V2", "V3")), _t("output", OUT, "float16", _O4)],
    (mul("Q0", "Q1"), "Q2", 1),
    _pcs(("B", U32, "Q0"), ("NH", U32, "Q1"), ("NK", U32, "K1"), ("T", U32, "Q2"), ("S", U32, "K2"),
         ("D", U32, "Q3")))
SDPA_DECODE_CACHE_F16 = _v(
    "sdpa_decode_cache_f16", "export", "ExportSdpaDecodeCacheF16Program",
    [_t("q", IN, "float16", ("B", "NH", "T", "D")), _t("k", IN, "float16", ("B", "NK", "S", "D"), role="state"),
     _t("v", IN, "float16", ("B", "NK", "S", "D"), role="state"), _t("output", OUT, "float16", ("B", "NH", "T", "D"))],
    ("NH", 1, 1),
    _pcs(("NH", U32, "NH"), ("NK", U32, "NK"), ("S", U32, "S"), ("D", U32, "D"),
         ("cache_position", U32, PushConstantInput("cache_position"))))
SDPA_DECODE_CACHE_WRITE_F32 = _v(
    "sdpa_decode_cache_write_f32", "optimized_qwen3", "SdpaDecodeCacheWriteF32Program",
    [_t("q", IN, "float16", ("B", "NH", "T", "D")), _t("new_k", IN, "float16", ("B", "NK", "T", "D")),
     _t("new_v", IN, "float16", ("B", "T", "NK", "D")), _t("k_cache", INOUT, "float16", ("B", "S", "NK", "D")),
     _t("v_cache", INOUT, "float16", ("B", "S", "NK", "D")), _t("output", OUT, "float16", ("B", "NH", "T", "D"))],
    ("NH", 1, 1),
    _pcs(("NH", U32, "NH"), ("NK", U32, "NK"), ("S", U32, "S"), ("D", U32, "D"),
         ("cache_position", U32, PushConstantInput("cache_position"))))

# ------------------------------------------------------------------ embedding / LM head / tokens
EMBEDDING_Q4_K_F32 = _v(
    "embedding_q4_k_f32", "export", "ExportEmbeddingQ4_KProgram",
    [_t("weight", IN, "uint32", ("V", 144), q4_k_words_layout(logical_k="H"), role="weight"),
     _t("indices", IN, "int64", ("I0", "I1")), _t("output", OUT, "float16", ("I0", "I1", "H"))],
    (ceil_div(mul(mul("I0", "I1"), "H"), 256), 1, 1),
    _pcs(("num_indices", U32, mul("I0", "I1")), ("embedding_dim", U32, "H")))
LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16 = _v(
    "lm_head_q6_k_argmax_partial_f16", "export", "LmHeadQ6KArgmaxPartialF16Program",
    [_t("x", IN, "float16", (1, 1, "K")), _wfield("weight", "q6_k", "N"),
     *_named_roles([_t("partial_scores", OUT, "float32", ("G",)), _t("partial_tokens", OUT, "uint32", ("G",))])],
    (ceil_div("N", 4), 1, 1), _pcs(("K", U32, "K"), ("N", U32, "N")))
QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32 = _v(
    "qwen3_token_select_reduce_chunks_f32", "export", "Qwen3TokenSelectReduceChunksF32Program",
    _named_roles([_t("scores", IN, "float32", ("G",)), _t("tokens", IN, "uint32", ("G",)),
                  _t("chunk_scores", OUT, "float32", ("C",)), _t("chunk_tokens", OUT, "uint32", ("C",))]),
    (ceil_div("G", 1024), 1, 1), _pcs(("G", U32, "G")))
QWEN3_TOKEN_SELECT_REDUCE_F32 = _v(
    "qwen3_token_select_reduce_f32", "export", "Qwen3TokenSelectReduceF32Program",
    _named_roles([_t("partial_scores", IN, "float32", ("G",)), _t("partial_tokens", IN, "uint32", ("G",)),
                  _t("eos_token_ids", IN, "int64", ("E",)), _t("next_token", OUT, "int64", (1, 1)),
                  _t("done", OUT, "uint32", (1,))]),
    (1, 1, 1), _pcs(("G", U32, "G"), ("E", U32, "E")))
QWEN3_TOKEN_STORE_EOS = _v(
    "qwen3_token_store_eos", "export", "Qwen3TokenStoreEosProgram",
    _named_roles([_t("next_token", IN, "int64", (1, 1)), _t("done", IN, "uint32", (1,)),
                  _t("generated_tokens", INOUT, "int64", (1, "G")), _t("generated_length", INOUT, "uint32", (1,)),
                  _t("stopped", INOUT, "uint32", (1,))]),
    (1, 1, 1), _pcs(("G", U32, "G"), ("stop_on_eos", U32, 1), ("token_index", U32, PushConstantInput("token_index"))))

# Permutation (output dim i reads input dim PERM[i]) of each ExportTransposeProgram
# variant; every transpose of the Qwen3 export swaps dims 1 and 2
# (quantized_qwen3/shaders/transpose_f32_*.py index in the order c0, c2, c1, c3).
TRANSPOSE_PERMUTATIONS: dict[str, tuple[int, ...]] = {
    "transpose_f32": (0, 2, 1, 3),
    # the Qwen3-ASR audio encoder's transposes (quantized_qwen3_asr/shaders/transpose_f32_*.py)
    "transpose_f32_d95ce920ac": (0, 2, 1),
    "transpose_f32_6a3397f037": (1, 0, 2),
    "transpose_f32_48d16b9b88": (0, 2, 1, 3),
    # OmniVoice's LLM (quantized_omnivoice/shaders/transpose_f32_*.py: heads <-> positions)
    "transpose_f32_322f87bdab": (0, 2, 1, 3),
    "transpose_f32_b4bb3205fc": (0, 2, 1, 3),
    "transpose_f32_e6f353739d": (0, 2, 1, 3),
}


def all_variants() -> dict[str, ShaderVariant]:
    return {v.name: v for v in globals().values() if isinstance(v, ShaderVariant)}

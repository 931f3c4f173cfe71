"""Drop-in conformance on the CPU (no kernels run).

1. Every op declaration in torch2vk_b200.runtime.variants equals the reference
   ShaderVariant of the same name: class_name, fields (name, io kind, role,
   dtype, symbolic shape, layout), push constants and dispatch grid.
2. The reference's own generated Qwen3 model code (models/quantized_qwen3 and
   models/optimized_qwen3: tensors/, dispatch/, shaders/) imported through
   torch2vk_b200.compat drives a prefill + decode step through RuntimeSession's
   validation; every contract class it dispatches has a CUDA op.
3. RuntimeSession.dispatch raises the reference dispatcher's errors.

Parts 1-2 read the reference sources and skip when they are absent.
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

import numpy as np
import pytest

# the reference checkout (read only): T2C_REFERENCE_ROOT, else a `reference` directory beside this
# repository's checkout; tests that need it skip where neither exists
REF_SRC = Path(os.environ.get("T2C_REFERENCE_ROOT", Path(__file__).resolve().parents[2] / "reference")) / "src"
needs_ref = pytest.mark.skipif(not (REF_SRC / "models" / "quantized_qwen3").is_dir(),
                               reason="reference sources not present")


@pytest.fixture()
def ref_modules():
    """Installs the torch2vk aliases and the reference `models` package; undoes both after."""
    saved = {k: v for k, v in sys.modules.items() if k == "torch2vk" or k.startswith(("torch2vk.", "models"))}
    for k in saved:
        del sys.modules[k]
    from torch2vk_b200 import compat

    compat.install()
    sys.path.append(str(REF_SRC))
    try:
        yield
    finally:
        sys.path.remove(str(REF_SRC))
        for k in [k for k in sys.modules if k == "torch2vk" or k.startswith(("torch2vk.", "models"))]:
            del sys.modules[k]
        sys.modules.update(saved)


def _variant_names():
    from torch2vk_b200.runtime import variants

    return sorted(variants.all_variants())


# The reference generator names transposes by a hash of their source; this one
# is the dim-1/2 swap that every transpose of the Qwen3 export uses.
REF_NAME = {"transpose_f32": "transpose_f32_9884b7b82d"}


@needs_ref
@pytest.mark.parametrize("name", _variant_names())
def test_variant_contract_matches_reference(ref_modules, name):
    from torch2vk_b200.runtime import variants

    ours = variants.all_variants()[name]
    if name == "rope_table_f32":
        pytest.skip("torch2vk.runtime.rope_table is itself aliased to this package")
    ref_name = REF_NAME.get(name, name)
    ref = None
    for pkg in ("models.quantized_qwen3.shaders", "models.optimized_qwen3.shaders"):
        try:
            ref = getattr(importlib.import_module(f"{pkg}.{ref_name}"), ref_name.upper())
            break
        except ModuleNotFoundError:
            continue
    assert ref is not None, f"no reference variant {ref_name}"
    a, b = ours.contract, ref.contract
    assert a.class_name == b.class_name
    assert a.fields == b.fields
    assert a.push_constants == b.push_constants
    assert a.dispatch == b.dispatch


def _drive_quantized_qwen3(rt, mt, cache_position):
    from models.quantized_qwen3.dispatch.decode_embed import run_decode_embed
    from models.quantized_qwen3.dispatch.decode_layer import run_decode_layer
    from models.quantized_qwen3.dispatch.decode_norm import run_decode_norm
    from models.quantized_qwen3.dispatch.embed_tokens import run_embed_tokens
    from models.quantized_qwen3.dispatch.text_layer import run_text_layer
    from models.quantized_qwen3.dispatch.text_norm import run_text_norm
    from models.quantized_qwen3.shaders.lm_head_q6_k_argmax_partial_f16 import LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16
    from models.quantized_qwen3.shaders.qwen3_token_select_reduce_chunks_f32 import (
        QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32,
    )
    from models.quantized_qwen3.shaders.qwen3_token_select_reduce_f32 import QWEN3_TOKEN_SELECT_REDUCE_F32
    from models.quantized_qwen3.shaders.qwen3_token_store_eos import QWEN3_TOKEN_STORE_EOS
    from models.quantized_qwen3.shaders.slice_last_token_f16 import SLICE_LAST_TOKEN_F16
    from torch2vk.runtime.rope_table import ROPE_TABLE_F32

    def head(x):
        LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16(rt, x=x, weight=mt.lm_head.p_weight, partial_scores=mt.lm_head_partial_scores,
                                        partial_tokens=mt.lm_head_partial_tokens)
        QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32(rt, scores=mt.lm_head_partial_scores, tokens=mt.lm_head_partial_tokens,
                                             chunk_scores=mt.lm_head_chunk_scores,
                                             chunk_tokens=mt.lm_head_chunk_tokens)
        QWEN3_TOKEN_SELECT_REDUCE_F32(rt, partial_scores=mt.lm_head_chunk_scores,
                                      partial_tokens=mt.lm_head_chunk_tokens, eos_token_ids=mt.eos_token_ids,
                                      next_token=mt.next_token, done=mt.done)

    def store(index):
        QWEN3_TOKEN_STORE_EOS(rt, next_token=mt.next_token, token_index=index, done=mt.done,
                              generated_tokens=mt.generated_tokens, generated_length=mt.generated_length,
                              stopped=mt.stopped)

    # the order of models/quantized_qwen3/run.py:_run_prefill and _run_decode_step
    with rt.frame("qwen3.prefill"):
        ROPE_TABLE_F32(rt, start_position=0, theta=1e6, cos=mt.prefill_rope.cos, sin=mt.prefill_rope.sin)
        run_embed_tokens(rt)
        for i in range(len(mt.text_layers)):
            run_text_layer(rt, i)
        run_text_norm(rt)
        SLICE_LAST_TOKEN_F16(rt, x=mt.text_norm.rms_norm, output=mt.prefill_lm_head_input)
        head(mt.prefill_lm_head_input)
        store(0)
    with rt.frame("qwen3.decode.0000"):
        ROPE_TABLE_F32(rt, start_position=cache_position, theta=1e6, cos=mt.decode_rope.cos, sin=mt.decode_rope.sin)
        run_decode_embed(rt)
        for i in range(len(mt.decode_layers)):
            run_decode_layer(rt, i, cache_position=cache_position)
        run_decode_norm(rt)
        head(mt.decode_norm.rms_norm)
        store(1)


@needs_ref
def test_reference_quantized_qwen3_dispatch_through_session(ref_modules):
    from models.quantized_qwen3.tensors.model import create_model_tensors
    from tests.dry_session import DrySession

    P = 8
    mt = create_model_tensors(prompt_length=P, max_sequence_length=64, num_hidden_layers=28, num_key_value_heads=8,
                              head_dim=128, max_new_tokens=4, eos_token_count=2, vocab_size=151936)
    rt = DrySession(mt)
    rt.initialize_session_tensors({mt.eos_token_ids: np.array([151643, 151645], np.int64)})
    zero = np.zeros((1, 8, 64, 128), np.float16)
    state = {c: zero for c in mt.key_caches + mt.value_caches}
    state.update({mt.generated_tokens: np.zeros((1, 4), np.int64), mt.generated_length: np.zeros(1, np.uint32),
                  mt.stopped: np.zeros(1, np.uint32)})
    with rt.request(inputs={mt.input_ids.name: np.zeros((1, P), np.int64),
                            mt.text_layers[0].cache_position.name: np.arange(P, dtype=np.int64)}, state=state):
        _drive_quantized_qwen3(rt, mt, cache_position=P)
    classes = {c for _, c, _, _ in rt.calls}
    assert classes <= set(rt._ops), classes - set(rt._ops)
    assert len(rt.calls) > 2000
    decode = [c for c in rt.calls if c[0] == "sdpa_decode_cache_f16"]
    assert len(decode) == 28 and all(c[3]["cache_position"] == P for c in decode)
    lin = [c for c in rt.calls if c[0] == "linear_nobias_q4_k_matvec_f32"]
    assert {c[2]["K"] for c in lin} == {1024, 2048, 3072}


@needs_ref
def test_replay_plan_of_reference_decode_frame(ref_modules):
    """rt.build_replay_plan over the reference's generated decode frame, then execute_replay with a new
    cache_position (models/quantized_qwen3/run.py replays its decode step this way): the plan re-issues
    the frame's dispatches in order, with the dynamic push constant substituted and nothing else changed."""
    from models.quantized_qwen3.tensors.model import create_model_tensors
    from tests.dry_session import DrySession
    from torch2vk.runtime.replay import execute_replay, stage_replay_step_inputs

    P = 8
    mt = create_model_tensors(prompt_length=P, max_sequence_length=64, num_hidden_layers=28, num_key_value_heads=8,
                              head_dim=128, max_new_tokens=4, eos_token_count=2, vocab_size=151936)
    rt = DrySession(mt)
    rt.initialize_session_tensors({mt.eos_token_ids: np.array([151643, 151645], np.int64)})
    zero = np.zeros((1, 8, 64, 128), np.float16)
    state = {c: zero for c in mt.key_caches + mt.value_caches}
    state.update({mt.generated_tokens: np.zeros((1, 4), np.int64), mt.generated_length: np.zeros(1, np.uint32),
                  mt.stopped: np.zeros(1, np.uint32)})
    with rt.request(inputs={mt.input_ids.name: np.zeros((1, P), np.int64),
                            mt.text_layers[0].cache_position.name: np.arange(P, dtype=np.int64)}, state=state):
        _drive_quantized_qwen3(rt, mt, cache_position=P)
        ctx = rt._frame_history["qwen3.decode.0000"]
        frame_calls = rt.calls[ctx.start_dispatch_index:ctx.end_dispatch_index]
        plan = rt.build_replay_plan(name="decode", frame="qwen3.decode.0000")
        assert plan.num_dispatches == len(frame_calls) > 300
        assert set(plan.dynamic_push_constant_names) == {"cache_position", "start_position", "theta", "token_index"}
        with pytest.raises(ValueError, match="unexpected dynamic push constants"):
            execute_replay(plan, dynamic_push_constants={"nope": 1})
        stage_replay_step_inputs(rt, plan=plan, inputs={})
        before = len(rt.calls)
        execute_replay(plan, dynamic_push_constants={"cache_position": P + 1, "token_index": 2})
        replayed = rt.calls[before:]
    assert [c[0] for c in replayed] == [c[0] for c in frame_calls]
    # the run scripts' cache helpers (models/quantized_qwen3/run.py imports them)
    from torch2vk.runtime.replay_cache_key import (
        build_cached_replay_plan,
        cached_replay_plan,
        replay_cache_namespace,
        source_tree_digest,
    )

    digest = source_tree_digest(REF_SRC / "models" / "quantized_qwen3" / "run.py")
    assert len(digest) == 16
    ns = replay_cache_namespace(name="decode", source_digest=digest, model_dir="/tmp", shape_key="p8")
    assert cached_replay_plan(rt, namespace=ns) is None
    built = build_cached_replay_plan(rt, namespace=ns, name="decode", frame="qwen3.decode.0000", readback_error="x")
    assert cached_replay_plan(rt, namespace=ns) is built
    for old, new in zip(frame_calls, replayed):
        assert new[2] == old[2]  # shape symbols
        want = dict(old[3])
        if "cache_position" in want and old[0].startswith(("sdpa_decode", "kv_cache_write_decode")):
            want["cache_position"] = P + 1
        if "token_index" in want:
            want["token_index"] = 2
        assert new[3] == want, old[0]


@needs_ref
def test_replay_plan_templates_across_sessions(ref_modules, tmp_path):
    """A cached plan written as an on-disk template (src/torch2vk/runtime/replay_cache.py) is found by a
    second session over freshly declared model tensors -- as another process would -- and replays the
    same dispatches there; a model with other shapes finds the template incompatible."""
    from models.quantized_qwen3.tensors.model import create_model_tensors
    from tests.dry_session import DrySession
    from torch2vk.runtime.replay import execute_replay, stage_replay_step_inputs
    from torch2vk.runtime.replay_cache_key import build_cached_replay_plan, cached_replay_plan

    P = 8

    def session(max_seq):
        mt = create_model_tensors(prompt_length=P, max_sequence_length=max_seq, num_hidden_layers=28,
                                  num_key_value_heads=8, head_dim=128, max_new_tokens=4, eos_token_count=2,
                                  vocab_size=151936)
        rt = DrySession(mt)
        rt.artifact_dir = tmp_path / "artifacts"
        rt.initialize_session_tensors({mt.eos_token_ids: np.array([151643, 151645], np.int64)})
        zero = np.zeros((1, 8, max_seq, 128), np.float16)
        state = {c: zero for c in mt.key_caches + mt.value_caches}
        state.update({mt.generated_tokens: np.zeros((1, 4), np.int64), mt.generated_length: np.zeros(1, np.uint32),
                      mt.stopped: np.zeros(1, np.uint32)})
        inputs = {mt.input_ids.name: np.zeros((1, P), np.int64),
                  mt.text_layers[0].cache_position.name: np.arange(P, dtype=np.int64)}
        return mt, rt, inputs, state

    ns = "decode:0123456789abcdef:/models/qwen3:p8"
    mt, rt, inputs, state = session(64)
    with rt.request(inputs=inputs, state=state):
        _drive_quantized_qwen3(rt, mt, cache_position=P)
        plan = build_cached_replay_plan(rt, namespace=ns, name="decode", frame="qwen3.decode.0000",
                                        readback_error="x")
    variants = {d.variant.name: d.variant for d in plan.dispatches}
    files = list((tmp_path / "replay_templates_v1").glob("*.pkl"))
    assert len(files) == 1

    # a second session over new LogicalTensor objects: the request's prefill runs as model code, the
    # decode step comes from the template (no plan was built in this session)
    mt2, rt2, inputs2, state2 = session(64)
    rt2._get_shader = variants.__getitem__
    with rt2.request(inputs=inputs2, state=state2):
        _drive_quantized_qwen3(rt2, mt2, cache_position=P)
        got = cached_replay_plan(rt2, namespace=ns)
        assert got is not None and got is not plan and got.session is rt2
        assert got.num_dispatches == plan.num_dispatches
        assert set(got.dynamic_push_constant_names) == set(plan.dynamic_push_constant_names)
        stage_replay_step_inputs(rt2, plan=got, inputs={})
        before = len(rt2.calls)
        execute_replay(got, dynamic_push_constants={"cache_position": P + 1, "token_index": 2})
        replayed = rt2.calls[before:]
    assert [c[0] for c in replayed] == [d.variant.name for d in plan.dispatches]
    assert all(c[2] == d.symbols for c, d in zip(replayed, plan.dispatches))

    # other shapes: the template does not match
    mt3, rt3, inputs3, state3 = session(128)
    rt3._get_shader = variants.__getitem__
    with rt3.request(inputs=inputs3, state=state3):
        with pytest.raises(RuntimeError, match="incompatible"):
            rt3.cached_replay_plans(ns)


@needs_ref
def test_reference_optimized_qwen3_decode_through_session(ref_modules):
    from models.optimized_qwen3.dispatch.decode_embed import run_decode_embed
    from models.optimized_qwen3.dispatch.decode_layer import run_decode_layer
    from models.optimized_qwen3.dispatch.decode_norm import run_decode_norm
    from models.optimized_qwen3.tensors.model import create_model_tensors
    from tests.dry_session import DrySession

    # sizes as models/optimized_qwen3/run.py derives them for an 8-token prompt
    mt = create_model_tensors(prompt_length=8, prefill_chunk_length=512, prefill_tail_length=8,
                              prefill_attention_length=64, max_sequence_length=192, num_hidden_layers=28,
                              num_key_value_heads=8, head_dim=128, max_new_tokens=4, eos_token_count=2,
                              vocab_size=151936)
    rt = DrySession(mt)
    state = {c: np.zeros(c.concrete_shape, np.float16) for c in mt.decode_key_caches + mt.decode_value_caches}
    state[mt.decode_rope.cos] = np.zeros((1, 1, 128), np.float16)
    state[mt.decode_rope.sin] = np.zeros((1, 1, 128), np.float16)
    state[mt.next_token] = np.zeros((1, 1), np.int64)
    with rt.request(state=state):
        with rt.frame("qwen3.decode.0000"):
            run_decode_embed(rt)
            for i in range(len(mt.decode_layers)):
                run_decode_layer(rt, i, cache_position=8)
            run_decode_norm(rt)
    classes = {c for _, c, _, _ in rt.calls}
    assert classes <= set(rt._ops), classes - set(rt._ops)
    assert "SdpaDecodeCacheWriteF32Program" in classes and "LinearNobiasQ4KQKVMatvecProgram" in classes or \
        "LinearNobiasQ4QKQ6VMatvecProgram" in classes


@needs_ref
def test_reference_optimized_qwen3_prefill_through_session(ref_modules):
    """The fp32-activation prefill chain (models/optimized_qwen3/run.py:394-445): full 512-token
    chunk + tail chunk, embedding, mask classifier, every layer, the last layer's decode-shaped tail,
    norm, LM head select and token store."""
    from models.optimized_qwen3.dispatch.embed_tokens import run_prefill_full_embed, run_prefill_tail_embed
    from models.optimized_qwen3.dispatch.text_layer import (
        run_prefill_full_layer,
        run_prefill_full_mask_opt,
        run_prefill_tail_last_layer_tail,
        run_prefill_tail_layer,
        run_prefill_tail_mask_opt,
    )
    from models.optimized_qwen3.dispatch.text_norm import run_text_norm
    from models.optimized_qwen3.shaders.lm_head_q6_k_argmax_partial_f16 import LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16
    from models.optimized_qwen3.shaders.qwen3_token_select_reduce_chunks_f32 import (
        QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32,
    )
    from models.optimized_qwen3.shaders.qwen3_token_select_reduce_f32 import QWEN3_TOKEN_SELECT_REDUCE_F32
    from models.optimized_qwen3.shaders.qwen3_token_store_eos_f32 import QWEN3_TOKEN_STORE_EOS_F32
    from models.optimized_qwen3.tensors.model import create_model_tensors
    from tests.dry_session import DrySession
    from torch2vk.runtime.rope_table import ROPE_TABLE_F32

    prompt, chunk = 520, 512
    tail, attn_len, max_seq = prompt - chunk, 576, 704
    mt = create_model_tensors(prompt_length=prompt, prefill_chunk_length=chunk, prefill_tail_length=tail,
                              prefill_attention_length=attn_len, max_sequence_length=max_seq, num_hidden_layers=28,
                              num_key_value_heads=8, head_dim=128, max_new_tokens=4, eos_token_count=1,
                              vocab_size=151936)
    rt = DrySession(mt)
    rt.initialize_session_tensors({mt.eos_token_ids: np.array([151645], np.int64)})
    caches = (mt.prefill_full_key_caches + mt.prefill_full_value_caches + mt.prefill_key_caches +
              mt.prefill_value_caches + mt.decode_key_caches + mt.decode_value_caches)
    state = {c: np.zeros(c.concrete_shape, np.float16) for c in caches}
    state.update({mt.generated_tokens: np.zeros((1, 4), np.int64), mt.generated_length: np.zeros(1, np.uint32),
                  mt.stopped: np.zeros(1, np.uint32)})
    inputs = {
        mt.prefill_full_input_ids.name: np.zeros((1, chunk), np.int64),
        mt.prefill_full_causal_mask.name: np.zeros((chunk, chunk), np.float16),
        mt.prefill_full_layers[0].cache_position.name: np.arange(chunk, dtype=np.int64),
        mt.prefill_tail_input_ids.name: np.zeros((1, tail), np.int64),
        mt.prefill_tail_causal_mask.name: np.zeros((tail, attn_len), np.float16),
        mt.prefill_tail_layers[0].cache_position.name: np.arange(chunk, prompt, dtype=np.int64),
    }
    with rt.request(inputs=inputs, state=state):
        with rt.frame("qwen3.prefill.full512"):
            ROPE_TABLE_F32(rt, start_position=0, theta=1e6, cos=mt.prefill_full_rope.cos, sin=mt.prefill_full_rope.sin)
            run_prefill_full_embed(rt)
            run_prefill_full_mask_opt(rt)
            for i in range(len(mt.prefill_full_layers)):
                run_prefill_full_layer(rt, i)
        with rt.frame("qwen3.prefill.tail"):
            ROPE_TABLE_F32(rt, start_position=chunk, theta=1e6, cos=mt.prefill_tail_rope.cos,
                           sin=mt.prefill_tail_rope.sin)
            run_prefill_tail_embed(rt)
            run_prefill_tail_mask_opt(rt)
            for i in range(len(mt.prefill_tail_layers) - 1):
                run_prefill_tail_layer(rt, i)
            run_prefill_tail_last_layer_tail(rt)
            run_text_norm(rt)
            # models/optimized_qwen3/run.py:116-139 (_run_lm_head_select)
            LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16(rt, x=mt.text_norm.mul_1, weight=mt.lm_head.p_weight,
                                            partial_scores=mt.lm_head_partial_scores,
                                            partial_tokens=mt.lm_head_partial_tokens)
            QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32(rt, scores=mt.lm_head_partial_scores,
                                                 tokens=mt.lm_head_partial_tokens,
                                                 chunk_scores=mt.lm_head_chunk_scores,
                                                 chunk_tokens=mt.lm_head_chunk_tokens)
            QWEN3_TOKEN_SELECT_REDUCE_F32(rt, partial_scores=mt.lm_head_chunk_scores,
                                          partial_tokens=mt.lm_head_chunk_tokens, eos_token_ids=mt.eos_token_ids,
                                          next_token=mt.next_token, done=mt.done)
            QWEN3_TOKEN_STORE_EOS_F32(rt, next_token=mt.next_token, token_index=0, done=mt.done,
                                      generated_tokens=mt.generated_tokens, generated_length=mt.generated_length,
                                      stopped=mt.stopped)
    classes = {c for _, c, _, _ in rt.calls}
    assert classes <= set(rt._ops), classes - set(rt._ops)
    for needed in ("LlamaMatmulQ4KF32Program", "LlamaFlashAttnF32F16F16Program", "OptimizedQwen3FaMaskOptF16Program",
                   "OptimizedQwen3RmsNormRopeTokenF32Program", "OptimizedQwen3TokenMajorValueCacheWriteF32ToF16PairProgram",
                   "SwigluF32Program", "AddF32PrefillProgram", "SliceLastTokenF32ToF16Program",
                   "OptimizedQwen3EmbeddingQ4KActF32Program"):
        assert needed in classes, needed
    fa = [c for c in rt.calls if c[1] == "LlamaFlashAttnF32F16F16Program"]
    assert len(fa) == 56 and {c[2]["T"] for c in fa} == {chunk, tail}


# ---------------------------------------------------------------- validation errors
def _tensors():
    from torch2vk_b200.runtime.logical import LogicalTensor, MemoryClass, TensorLifetime, TensorRole
    from torch2vk_b200.runtime.types import TensorSpec, q4_k_words_layout

    def t(name, dtype, shape, role=TensorRole.ACTIVATION, **kw):
        mem = {TensorRole.ACTIVATION: MemoryClass.FRAME_WORKSPACE, TensorRole.INPUT: MemoryClass.HOST_INPUT,
               TensorRole.WEIGHT: MemoryClass.MODEL_WEIGHT}[role]
        life = TensorLifetime.MODEL if role is TensorRole.WEIGHT else TensorLifetime.FRAME
        return LogicalTensor(spec=TensorSpec(dtype, shape), role=role, memory=mem, lifetime=life, name=name, **kw)

    x = t("x", "float16", (1, 2, 512), TensorRole.INPUT)
    w = t("w", "uint32", (256, 72), TensorRole.WEIGHT, checkpoint_key="w", layout=q4_k_words_layout(logical_k=512))
    y = t("y", "float16", (1, 2, 256))
    return t, x, w, y


def test_dispatch_validation_errors():
    from tests.dry_session import DrySession
    from torch2vk_b200.runtime import variants as V
    from torch2vk_b200.runtime.logical import bind_logical_tensor_alias

    t, x, w, y = _tensors()
    rt = DrySession()
    rt.register_host_inputs({x: np.zeros((1, 2, 512), np.float16)})
    with pytest.raises(RuntimeError, match="active rt.frame"):
        V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=x, weight=w, output=y)
    with rt.frame("f"):
        with pytest.raises(ValueError, match="missing tensor fields"):
            V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=x, weight=w)
        with pytest.raises(ValueError, match="unexpected fields"):
            V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=x, weight=w, output=y, bias=y)
        with pytest.raises(ValueError, match="missing push constant inputs"):
            V.SDPA_DECODE_CACHE_F16(rt, q=y, k=y, v=y, output=y)
        with pytest.raises(TypeError, match="expects LogicalTensor"):
            V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=np.zeros(3), weight=w, output=y)
        with pytest.raises(ValueError, match="expects dtype"):
            V.LINEAR_NOBIAS_Q6_K_MATVEC_F32(rt, x=x, weight=w, output=y)
        bad_y = t("bad_y", "float16", (1, 3, 256))
        with pytest.raises(ValueError, match="Shape symbol X1 bound to both"):
            V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=x, weight=w, output=bad_y)
        bad_w = t("bad_w", "uint32", (256, 36), checkpoint_key="bw", role=__import__(
            "torch2vk_b200.runtime.logical", fromlist=["TensorRole"]).TensorRole.WEIGHT,
            layout=__import__("torch2vk_b200.runtime.types", fromlist=["q4_k_words_layout"]).q4_k_words_layout(
                logical_k=512))
        with pytest.raises(ValueError, match="expects dim"):
            V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=x, weight=bad_w, output=y)
        z = t("z", "float16", (1, 2, 256))
        with pytest.raises(RuntimeError, match="cannot be read before"):
            V.ADD_F32_18(rt, x=z, y=z, output=y)
        V.LINEAR_NOBIAS_Q4_K_MATVEC_F32(rt, x=x, weight=w, output=y)
        view = t("view", "float16", (1, 2, 256))
        bind_logical_tensor_alias(y, view)
        with pytest.raises(RuntimeError, match="cannot be written"):
            V.ADD_F32_18(rt, x=y, y=y, output=view)
        assert rt.dispatch_records[-1].shader == "linear_nobias_q4_k_matvec_f32"
        assert y.writer is not None and y.writer.shader == "linear_nobias_q4_k_matvec_f32"
    assert y.buffer is None  # frame workspace released at frame exit
    with pytest.raises(ValueError, match="byte size differs"):
        bind_logical_tensor_alias(y, t("small", "float16", (1, 2, 2)))


def test_declaration_rules():
    from torch2vk_b200.runtime.logical import LogicalTensor, MemoryClass, TensorLifetime, TensorRole
    from torch2vk_b200.runtime.types import TensorSpec

    w = LogicalTensor(spec=TensorSpec("uint32", (4, 36)), role=TensorRole.WEIGHT, memory=MemoryClass.MODEL_WEIGHT,
                      lifetime=TensorLifetime.MODEL, name="w")
    with pytest.raises(ValueError, match="checkpoint_key"):
        w.validate_declaration()
    a = LogicalTensor(spec=TensorSpec("float16", (4,)), role=TensorRole.ACTIVATION,
                      memory=MemoryClass.REQUEST_STATE, lifetime=TensorLifetime.FRAME, name="a")
    with pytest.raises(ValueError, match="FRAME_WORKSPACE"):
        a.validate_declaration()
    with pytest.raises(RuntimeError, match="runtime state"):
        a.buffer = object()


@needs_ref
def test_reference_asr_audio_encoder_dispatch_through_session(ref_modules):
    """The reference's generated Qwen3-ASR audio tower (models/quantized_qwen3_asr/dispatch/audio_encoder.py)
    for 3000 mel frames (30 chunks, 390 tokens) through RuntimeSession's validation: every contract class
    it dispatches (Q8_0 conv2d / linear with bias, GELU, LayerNorm, masked SDPA, transposes, gather) has
    a CUDA op, and the transposes have known permutations."""
    from models.quantized_qwen3_asr.dispatch.audio_encoder import run_audio_encoder
    from models.quantized_qwen3_asr.tensors.model import create_model_tensors
    from tests.dry_session import DrySession
    from torch2vk_b200.runtime.variants import TRANSPOSE_PERMUTATIONS

    frames, chunks, tokens, prompt = 3000, 30, 390, 400
    mt = create_model_tensors(input_ids_shape=(1, prompt), attention_mask_shape=(1, prompt),
                              input_features_shape=(1, 128, frames), feature_attention_mask_shape=(1, frames),
                              prompt_length=prompt, audio_chunk_count=chunks, audio_sequence_length=tokens,
                              max_sequence_length=prompt + 16, num_hidden_layers=28, num_key_value_heads=8,
                              head_dim=128, max_new_tokens=4, eos_token_count=2, vocab_size=151936)
    ae = mt.audio_encoder
    rt = DrySession(mt)
    inputs = {ae.x.name: np.zeros(ae.x.spec.shape, np.float16),
              ae.position_embedding.name: np.zeros(ae.position_embedding.spec.shape, np.float16),
              ae.compact_index.name: np.arange(tokens, dtype=np.int64),
              ae.attention_mask.name: np.zeros(ae.attention_mask.spec.shape, np.float16)}
    with rt.request(inputs=inputs):
        with rt.frame("spike.audio"):
            run_audio_encoder(rt)
    classes = {c for _, c, _, _ in rt.calls}
    assert classes <= set(rt._ops), classes - set(rt._ops)
    assert {"ExportConv2dQ8_0WeightF32BiasProgram", "ExportLinearBiasQ8_0WeightF32BiasProgram",
            "ExportSdpaProgram", "ExportLayerNormF32WeightF32BiasProgram"} <= classes
    for name, cls, _, _ in rt.calls:
        if cls == "ExportTransposeProgram":
            assert name in TRANSPOSE_PERMUTATIONS, name
    sdpa = [c for c in rt.calls if c[1] == "ExportSdpaProgram"]
    assert len(sdpa) == 18 and all(c[3]["D"] == 64 and c[3]["T"] == tokens for c in sdpa)


@needs_ref
def test_reference_asr_text_decoder_through_session(ref_modules):
    """The Qwen3-ASR pipeline after the audio tower (models/quantized_qwen3_asr/run.py:366-470): RoPE
    table, Q8_0 token embedding, audio-feature injection (index copy), 28 text layers, norm, last-token
    slice, LM head select, ASR token store, then one decode step; every class has a CUDA op."""
    from models.quantized_qwen3_asr.dispatch.audio_encoder import run_audio_encoder
    from models.quantized_qwen3_asr.dispatch.audio_inject import run_audio_inject
    from models.quantized_qwen3_asr.dispatch.decode_embed import run_decode_embed
    from models.quantized_qwen3_asr.dispatch.decode_layer import run_decode_layer
    from models.quantized_qwen3_asr.dispatch.decode_norm import run_decode_norm
    from models.quantized_qwen3_asr.dispatch.embed_tokens import run_embed_tokens
    from models.quantized_qwen3_asr.dispatch.text_layer import run_text_layer
    from models.quantized_qwen3_asr.dispatch.text_norm import run_text_norm
    from models.quantized_qwen3_asr.shaders.lm_head_q6_k_argmax_partial_f16 import LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16
    from models.quantized_qwen3_asr.shaders.qwen3_asr_token_store_eos import QWEN3_ASR_TOKEN_STORE_EOS
    from models.quantized_qwen3_asr.shaders.qwen3_token_select_reduce_chunks_f32 import (
        QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32,
    )
    from models.quantized_qwen3_asr.shaders.qwen3_token_select_reduce_f32 import QWEN3_TOKEN_SELECT_REDUCE_F32
    from models.quantized_qwen3_asr.shaders.slice_last_token_f16 import SLICE_LAST_TOKEN_F16
    from models.quantized_qwen3_asr.tensors.model import create_model_tensors
    from tests.dry_session import DrySession
    from torch2vk.runtime.rope_table import run_rope_table_f32

    frames, chunks, tokens, prompt = 3000, 30, 390, 400
    mt = create_model_tensors(input_ids_shape=(1, prompt), attention_mask_shape=(1, prompt),
                              input_features_shape=(1, 128, frames), feature_attention_mask_shape=(1, frames),
                              prompt_length=prompt, audio_chunk_count=chunks, audio_sequence_length=tokens,
                              max_sequence_length=prompt + 16, num_hidden_layers=28, num_key_value_heads=8,
                              head_dim=128, max_new_tokens=4, eos_token_count=2, vocab_size=151936)

    def _run_lm_head_select(rt, *, x):  # run.py:73-96
        LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16(rt, x=x, weight=mt.lm_head.p_weight, partial_scores=mt.lm_head_partial_scores,
                                        partial_tokens=mt.lm_head_partial_tokens)
        QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32(rt, scores=mt.lm_head_partial_scores, tokens=mt.lm_head_partial_tokens,
                                             chunk_scores=mt.lm_head_chunk_scores,
                                             chunk_tokens=mt.lm_head_chunk_tokens)
        QWEN3_TOKEN_SELECT_REDUCE_F32(rt, partial_scores=mt.lm_head_chunk_scores,
                                      partial_tokens=mt.lm_head_chunk_tokens, eos_token_ids=mt.eos_token_ids,
                                      next_token=mt.next_token, done=mt.done)

    def _slice_prefill_lm_head_input(rt):  # run.py:99-105
        SLICE_LAST_TOKEN_F16(rt, x=mt.text_norm.rms_norm, output=mt.prefill_lm_head_input)

    ae = mt.audio_encoder
    rt = DrySession(mt)
    rt.initialize_session_tensors({mt.eos_token_ids: np.array([151643, 151645], np.int64)})
    inputs = {ae.x.name: np.zeros(ae.x.spec.shape, np.float16),
              ae.position_embedding.name: np.zeros(ae.position_embedding.spec.shape, np.float16),
              ae.compact_index.name: np.arange(tokens, dtype=np.int64),
              ae.attention_mask.name: np.zeros(ae.attention_mask.spec.shape, np.float16),
              "input_ids": np.zeros((1, prompt), np.int64),
              mt.position_ids.name: np.zeros((3, 1, prompt), np.int64),
              mt.audio_inject.audio_positions.name: np.arange(5, 5 + tokens, dtype=np.int64),
              mt.text_layers[0].cache_position.name: np.arange(prompt, dtype=np.int64)}
    zero = np.zeros((1, 8, prompt + 16, 128), np.float16)
    state = {c: zero for c in mt.key_caches + mt.value_caches}
    state.update({mt.generated_tokens: np.zeros((1, 4), np.int64), mt.generated_length: np.zeros(1, np.uint32),
                  mt.stopped: np.zeros(1, np.uint32)})
    with rt.request(inputs=inputs, state=state):
        with rt.frame("spike.audio"):
            run_audio_encoder(rt)
        run_rope_table_f32(rt, start_position=0, theta=1e6, cos=mt.prefill_rope.cos, sin=mt.prefill_rope.sin,
                           frame_name="spike.text.prefill_rope")
        with rt.frame("spike.text.prefill"):
            run_embed_tokens(rt)
            run_audio_inject(rt)
            for i in range(len(mt.text_layers)):
                run_text_layer(rt, i)
            run_text_norm(rt)
            _slice_prefill_lm_head_input(rt)
            _run_lm_head_select(rt, x=mt.prefill_lm_head_input)
        with rt.frame("spike.text.token_store"):
            QWEN3_ASR_TOKEN_STORE_EOS(rt, next_token=mt.next_token, token_index=0, done=mt.done,
                                      generated_tokens=mt.generated_tokens, generated_length=mt.generated_length,
                                      stopped=mt.stopped)
        run_rope_table_f32(rt, start_position=prompt, theta=1e6, cos=mt.decode_rope.cos, sin=mt.decode_rope.sin,
                           frame_name="spike.decode.rope.0000")
        with rt.frame("spike.decode.0000"):
            run_decode_embed(rt)
            for i in range(len(mt.decode_layers)):
                run_decode_layer(rt, i, cache_position=prompt)
            run_decode_norm(rt)
            _run_lm_head_select(rt, x=mt.decode_norm.rms_norm)
            QWEN3_ASR_TOKEN_STORE_EOS(rt, next_token=mt.next_token, token_index=1, done=mt.done,
                                      generated_tokens=mt.generated_tokens, generated_length=mt.generated_length,
                                      stopped=mt.stopped)
    classes = {c for _, c, _, _ in rt.calls}
    assert classes <= set(rt._ops), classes - set(rt._ops)
    assert {"ExportEmbeddingQ8_0Program", "ExportIndexCopyF32Program", "Qwen3AsrTokenStoreEosProgram",
            "ExportSdpaDecodeCacheF16Program"} <= classes


@needs_ref
def test_reference_optimized_asr_text_decoder_through_session(ref_modules):
    """models/optimized_qwen3_asr (run.py:369-420 and its decode step :140-161): audio tower, prefill with
    the fused Q4_K pair / triple linears, cache-writing attention, the last layer's tail, norm, LM head
    select and ASR token store, then one decode step with the cache-writing decode attention.  The
    package's __init__ pulls the forced aligner's audio dependencies (absent here), so the package
    module is registered without it; its generated tensors / dispatch / shaders modules import as is."""
    import types

    pkg = types.ModuleType("models.optimized_qwen3_asr")
    pkg.__path__ = [str(REF_SRC / "models" / "optimized_qwen3_asr")]
    import models

    sys.modules["models.optimized_qwen3_asr"] = pkg
    from models.optimized_qwen3_asr.dispatch.audio_encoder import run_audio_encoder
    from models.optimized_qwen3_asr.dispatch.audio_inject import run_audio_inject
    from models.optimized_qwen3_asr.dispatch.decode_embed import run_decode_embed
    from models.optimized_qwen3_asr.dispatch.decode_layer import run_decode_layer
    from models.optimized_qwen3_asr.dispatch.decode_norm import run_decode_norm
    from models.optimized_qwen3_asr.dispatch.embed_tokens import run_embed_tokens
    from models.optimized_qwen3_asr.dispatch.text_layer import run_text_last_layer_tail, run_text_layer
    from models.optimized_qwen3_asr.dispatch.text_norm import run_text_norm
    from models.optimized_qwen3_asr.shaders.lm_head_q6_k_argmax_partial_f16 import LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16
    from models.optimized_qwen3_asr.shaders.qwen3_asr_token_store_eos import QWEN3_ASR_TOKEN_STORE_EOS
    from models.optimized_qwen3_asr.shaders.qwen3_token_select_reduce_chunks_f32 import (
        QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32,
    )
    from models.optimized_qwen3_asr.shaders.qwen3_token_select_reduce_f32 import QWEN3_TOKEN_SELECT_REDUCE_F32
    from models.optimized_qwen3_asr.tensors.model import create_model_tensors
    from tests.dry_session import DrySession
    from torch2vk.runtime.rope_table import ROPE_TABLE_F32, run_rope_table_f32

    assert models is not None
    frames, chunks, tokens, prompt = 3000, 30, 390, 400
    mt = create_model_tensors(input_ids_shape=(1, prompt), attention_mask_shape=(1, prompt),
                              input_features_shape=(1, 128, frames), feature_attention_mask_shape=(1, frames),
                              prompt_length=prompt, audio_chunk_count=chunks, audio_sequence_length=tokens,
                              max_sequence_length=prompt + 16, num_hidden_layers=28, num_key_value_heads=8,
                              head_dim=128, max_new_tokens=4, eos_token_count=2, vocab_size=151936)

    def head(x):  # run.py:104-127
        LM_HEAD_Q6_K_ARGMAX_PARTIAL_F16(rt, x=x, weight=mt.lm_head.p_weight, partial_scores=mt.lm_head_partial_scores,
                                        partial_tokens=mt.lm_head_partial_tokens)
        QWEN3_TOKEN_SELECT_REDUCE_CHUNKS_F32(rt, scores=mt.lm_head_partial_scores, tokens=mt.lm_head_partial_tokens,
                                             chunk_scores=mt.lm_head_chunk_scores,
                                             chunk_tokens=mt.lm_head_chunk_tokens)
        QWEN3_TOKEN_SELECT_REDUCE_F32(rt, partial_scores=mt.lm_head_chunk_scores,
                                      partial_tokens=mt.lm_head_chunk_tokens, eos_token_ids=mt.eos_token_ids,
                                      next_token=mt.next_token, done=mt.done)

    def store(i):
        QWEN3_ASR_TOKEN_STORE_EOS(rt, next_token=mt.next_token, token_index=i, done=mt.done,
                                  generated_tokens=mt.generated_tokens, generated_length=mt.generated_length,
                                  stopped=mt.stopped)

    ae = mt.audio_encoder
    rt = DrySession(mt)
    rt.initialize_session_tensors({mt.eos_token_ids: np.array([151643, 151645], np.int64)})
    inputs = {ae.x.name: np.zeros(ae.x.spec.shape, np.float16),
              ae.position_embedding.name: np.zeros(ae.position_embedding.spec.shape, np.float16),
              ae.compact_index.name: np.arange(tokens, dtype=np.int64),
              ae.attention_mask.name: np.zeros(ae.attention_mask.spec.shape, np.float16),
              "input_ids": np.zeros((1, prompt), np.int64),
              mt.position_ids.name: np.zeros((3, 1, prompt), np.int64),
              mt.audio_inject.audio_positions.name: np.arange(5, 5 + tokens, dtype=np.int64),
              mt.text_layers[0].cache_position.name: np.arange(prompt, dtype=np.int64)}
    zero = np.zeros((1, 8, prompt + 16, 128), np.float16)
    state = {c: zero for c in mt.key_caches + mt.value_caches}
    state.update({mt.generated_tokens: np.zeros((1, 4), np.int64), mt.generated_length: np.zeros(1, np.uint32),
                  mt.stopped: np.zeros(1, np.uint32)})
    with rt.request(inputs=inputs, state=state):
        with rt.frame("spike.audio"):
            run_audio_encoder(rt)
        run_rope_table_f32(rt, start_position=0, theta=1e6, cos=mt.prefill_rope.cos, sin=mt.prefill_rope.sin,
                           frame_name="spike.text.prefill_rope")
        with rt.frame("spike.text.prefill"):
            run_embed_tokens(rt)
            run_audio_inject(rt)
            for i in range(len(mt.text_layers) - 1):
                run_text_layer(rt, i)
            run_text_last_layer_tail(rt)
            run_text_norm(rt)
            head(mt.text_norm.mul_1)
            store(0)
        with rt.frame("spike.decode.0000"):
            ROPE_TABLE_F32(rt, start_position=prompt, theta=1e6, cos=mt.decode_rope.cos, sin=mt.decode_rope.sin)
            run_decode_embed(rt)
            for i in range(len(mt.decode_layers)):
                run_decode_layer(rt, i, cache_position=prompt)
            run_decode_norm(rt)
            head(mt.decode_norm.mul_1)
            store(1)
    classes = {c for _, c, _, _ in rt.calls}
    assert classes <= set(rt._ops), classes - set(rt._ops)
    assert {"LinearNobiasQ4KPairProgram", "LinearNobiasQ4KTripleProgram", "OptimizedQwen3SdpaCausalCacheWriteProgram",
            "SdpaDecodeCacheWriteF16Program", "Qwen3AsrTokenStoreEosProgram"} <= classes, classes


@pytest.mark.skipif(not (REF_SRC / "models" / "quantized_omnivoice").is_dir(), reason="reference sources not present")
def test_reference_omnivoice_llm_step_through_session(ref_modules):
    """The reference's generated OmniVoice generation step up to the audio heads
    (models/quantized_omnivoice/run.py:113-129: input embedding, dispatch/llm_forward.py, dispatch/audio_head.py)
    through RuntimeSession's validation: every contract class it dispatches has a CUDA op (the Q8_0 input
    embedding, Q4_K / Q6_K linears, RMSNorms, the unfused RoPE chain, bidirectional masked GQA SDPA at D = 128),
    and every transpose has a known permutation.  CFG scoring and the top-k token update are not served."""
    from models.quantized_omnivoice.dispatch.audio_head import run_audio_head
    from models.quantized_omnivoice.dispatch.llm_forward import run_llm_forward
    from models.quantized_omnivoice.shaders.omnivoice_input_embed_q8_0_f32 import OMNIVOICE_INPUT_EMBED_Q8_0_F32
    from models.quantized_omnivoice.tensors.model import create_model_tensors, model_tensors
    from torch2vk.runtime.rope_table import run_rope_table_f32
    from tests.dry_session import DrySession
    from torch2vk_b200.runtime.variants import TRANSPOSE_PERMUTATIONS

    create_model_tensors(target_len=40)
    mt = model_tensors()
    rt = DrySession(mt)
    S = mt.batch_input_ids.spec.shape[2]
    state = {mt.batch_input_ids: np.zeros((2, 8, S), np.int64), mt.batch_audio_mask: np.zeros((2, S), np.uint32),
             mt.attention_mask: np.zeros((2, 1, S, S), np.float16), mt.tokens: np.zeros((1, 8, 40), np.int64)}
    with rt.request(state=state):
        # run.py:62-101 (_run_rope_table, _run_input_embed), restated: run.py itself imports audio I/O modules
        run_rope_table_f32(rt, start_position=0, theta=1_000_000.0, cos=mt.rope.cos, sin=mt.rope.sin,
                           frame_name="omnivoice.rope")
        with rt.frame("omnivoice.step.0000"):
            OMNIVOICE_INPUT_EMBED_Q8_0_F32(rt, text_weight=mt.text_embedding_weight,
                                           audio_weight=mt.audio_embedding_weight,
                                           batch_input_ids=mt.batch_input_ids, batch_audio_mask=mt.batch_audio_mask,
                                           hidden_states=mt.llm_forward.hidden_states)
            run_llm_forward(rt)
            run_audio_head(rt)
    classes = {c for _, c, _, _ in rt.calls}
    assert classes <= set(rt._ops), classes - set(rt._ops)
    assert {"OmniVoiceInputEmbedQ8_0Program", "ExportSdpaProgram", "ExportLinearNobiasQ6KProgram"} <= classes
    for name, cls, _, _ in rt.calls:
        if cls == "ExportTransposeProgram":
            assert name in TRANSPOSE_PERMUTATIONS, name
    sdpa = [c for c in rt.calls if c[1] == "ExportSdpaProgram"]
    assert len(sdpa) == 28 and all(c[3]["D"] == 128 and c[3]["NH"] == 16 and c[3]["NK"] == 8 for c in sdpa)

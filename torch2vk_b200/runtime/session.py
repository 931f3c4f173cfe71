"""RuntimeSession for the CUDA backend: the drop-in for torch2vk.runtime.session.RuntimeSession
(src/torch2vk/runtime/session.py:77-631 with dispatcher.py:28-172 and materialization.py).

Same surface and rules: request / frame scopes, dispatch only inside a frame,
contract validation (missing / extra fields, push-constant inputs, dtype,
rank, shape-symbol binding, layout), materialization by memory class
(weights from the GGUF checkpoint by checkpoint_key, host inputs, request
state, frame workspace released at frame exit), readback, dispatch records.
Underneath, every dispatch resolves `variant.contract.class_name` in the CUDA
op table (torch2vk_b200.runtime.optable) and launches libt2c_sm100 kernels on
the session's CUDA stream.  There is no CPU fallback: a contract without a
CUDA op raises.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence
from contextlib import contextmanager
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

from torch2vk_b200.gguf import GGUFFile
from torch2vk_b200.runtime.logical import (
    DispatchWriter,
    LogicalTensor,
    MemoryClass,
    TensorLifetime,
    TensorRole,
    collect_named_logical_tensors,
)
from torch2vk_b200.runtime.shader import (
    DispatchRecord,
    DTypeReference,
    IOKind,
    PushConstantInput,
    ShaderVariant,
    TensorFieldSpec,
    eval_expr,
)
from torch2vk_b200.runtime.replay import (
    ReplayDispatch,
    ReplayPlan,
    build_replay_plan_impl,
    push_inputs_of,
    rebind_replay_plan_impl,
    replay_plan_compatible_impl,
)
from torch2vk_b200.runtime.types import bind_tensor_layout_symbols, concrete_shape, tensor_nbytes

TORCH_DTYPES = {
    "float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16, "int8": torch.int8,
    "uint8": torch.uint8, "int16": torch.int16, "uint16": torch.uint16, "int32": torch.int32,
    "uint32": torch.uint32, "int64": torch.int64, "float64": torch.float64, "bool": torch.int32,
}
NUMPY_DTYPES = {"bool": np.uint32}


@dataclass
class FrameContext:
    frame: str
    start_dispatch_index: int
    end_dispatch_index: int
    used_tensors: list[LogicalTensor] = field(default_factory=list)
    written_tensors: list[LogicalTensor] = field(default_factory=list)
    registered_inputs: list[LogicalTensor] = field(default_factory=list)


class RuntimeSession:
    """Owns device memory for LogicalTensors and dispatches contracts to sm_100a kernels."""

    def __init__(self, *, device_index: int = 0, artifact_dir: str | Path | None = None,
                 model_dir: str | Path | None = None, profile_dir: str | Path | None = None,
                 model_tensors: object | None = None, session_tensors: Mapping[LogicalTensor, object] | None = None,
                 get_shader: Callable[[str], ShaderVariant] | None = None) -> None:
        if not torch.cuda.is_available():
            raise RuntimeError("RuntimeSession needs a CUDA device (sm_100a); there is no CPU fallback")
        self.device = torch.device("cuda", device_index)
        self.stream = torch.cuda.Stream(device=self.device)
        self.artifact_dir = None if artifact_dir is None else Path(artifact_dir).expanduser().resolve()
        self.model_dir = None if model_dir is None else Path(model_dir).expanduser().resolve()
        self.profile_dir = profile_dir
        if model_tensors is not None:
            collect_named_logical_tensors(model_tensors)
        self._model_tensors = model_tensors
        self._get_shader = get_shader
        self._inputs: dict[LogicalTensor, object] = {}
        self._request_active = False
        self._frame_stack: list[FrameContext] = []
        self._frame_history: dict[str, FrameContext] = {}
        self._dispatch_records: list[DispatchRecord] = []
        self._checkpoints: dict[Path, GGUFFile] = {}
        self._weight_cache: dict[str, torch.Tensor] = {}
        self._request_tensors: set[LogicalTensor] = set()
        self._frame_tensors: list[LogicalTensor] = []
        self._closed = False
        from torch2vk_b200.runtime import optable  # the CUDA op table (loads libt2c_sm100.so)

        self._ops = optable.OPS
        if session_tensors:
            self.initialize_session_tensors(session_tensors)

    @classmethod
    def open(cls, **kwargs) -> "RuntimeSession":
        return cls(**kwargs)

    def __enter__(self) -> "RuntimeSession":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    # ----------------------------------------------------------- properties
    @property
    def dispatch_records(self) -> tuple[DispatchRecord, ...]:
        return tuple(self._dispatch_records)

    @property
    def model_tensors(self) -> object | None:
        return self._model_tensors

    # ---------------------------------------------------------------- scopes
    @contextmanager
    def request(self, *, inputs: Mapping[str, object] | None = None, state: Mapping[LogicalTensor, object] | None = None):
        self._require_open()
        if self._request_active:
            raise RuntimeError("RuntimeSession.request cannot be nested")
        self._request_active = True
        try:
            if inputs:
                named = self._named_model_tensors()
                bound = {}
                for name, value in inputs.items():
                    if name not in named:
                        raise KeyError(f"request input {name!r} is not a named model tensor")
                    bound[named[name]] = value
                self.register_host_inputs(bound)
            if state:
                for tensor, value in state.items():
                    tensor.validate_declaration()
                    if tensor.role is not TensorRole.STATE and tensor.memory is not MemoryClass.REQUEST_STATE:
                        raise ValueError(f"{tensor.name} is not request state")
                    self._upload(tensor, value)
                    self._request_tensors.add(tensor)
            yield self
        finally:
            try:
                self.synchronize()
                for tensor in self._request_tensors:
                    self._drop(tensor)
                self._request_tensors.clear()
                self._inputs.clear()
            finally:
                self._request_active = False

    @contextmanager
    def frame(self, name: str):
        if not name:
            raise ValueError("frame name must be non-empty")
        ctx = FrameContext(frame=name, start_dispatch_index=len(self._dispatch_records),
                           end_dispatch_index=len(self._dispatch_records))
        self._frame_stack.append(ctx)
        try:
            yield ctx
            ctx.end_dispatch_index = len(self._dispatch_records)
        finally:
            popped = self._frame_stack.pop()
            if popped is not ctx:
                raise RuntimeError("RuntimeSession frame stack corrupted")
            self._frame_history[ctx.frame] = ctx
            self.synchronize()
            self._release_frame_tensors()

    # ---------------------------------------------------------------- inputs
    def register_host_inputs(self, inputs: Mapping[LogicalTensor, object]) -> None:
        for tensor, value in inputs.items():
            if not isinstance(tensor, LogicalTensor):
                raise TypeError(f"register_host_inputs key must be LogicalTensor, got {type(tensor).__name__}")
            tensor.validate_declaration()
            if tensor.role is not TensorRole.INPUT:
                raise ValueError(f"{tensor.name} is not an input tensor")
            if tensor.memory is MemoryClass.SESSION_TENSOR:
                raise ValueError(f"{tensor.name} is a session tensor; use initialize_session_tensors(...)")
            self._inputs[tensor] = value
            self._drop(tensor)
            if self._frame_stack:
                self._frame_stack[-1].registered_inputs.append(tensor)

    def release_host_inputs(self, tensors: Sequence[LogicalTensor]) -> None:
        for tensor in tensors:
            if tensor.lifetime not in {TensorLifetime.FRAME, TensorLifetime.OP}:
                raise ValueError(f"{tensor.name} is not a frame-local host input")
            self._inputs.pop(tensor, None)
            self._drop(tensor)

    def initialize_session_tensors(self, tensors: Mapping[LogicalTensor, object]) -> None:
        self._require_open()
        for tensor, value in tensors.items():
            tensor.validate_declaration()
            if tensor.role is not TensorRole.INPUT or tensor.memory is not MemoryClass.SESSION_TENSOR:
                raise ValueError(f"{tensor.name} is not a session tensor input")
            if tensor.buffer is not None:
                raise RuntimeError(f"{tensor.name} session tensor is already registered")
            self._upload(tensor, value)

    # ------------------------------------------------------------- weights
    def materialize_model_weights(self) -> None:
        if self._model_tensors is None:
            raise RuntimeError("RuntimeSession has no model_tensors to materialize")
        for tensor in collect_named_logical_tensors(self._model_tensors).values():
            if tensor.role is TensorRole.WEIGHT:
                self._materialize_weight(tensor)

    def _checkpoint(self, tensor: LogicalTensor) -> GGUFFile:
        if self.model_dir is None:
            raise RuntimeError(f"{tensor.name}: RuntimeSession.open(..., model_dir=...) is required for weights")
        path = Path(tensor.checkpoint).expanduser() if tensor.checkpoint else self.model_dir / "model.gguf"
        if not path.is_absolute():
            path = self.model_dir / path
        path = path.resolve()
        if path not in self._checkpoints:
            if path.suffix != ".gguf":
                raise RuntimeError(f"{tensor.name}: only GGUF checkpoints are supported, got {path}")
            self._checkpoints[path] = GGUFFile(path)
        return self._checkpoints[path]

    def _materialize_weight(self, tensor: LogicalTensor) -> None:
        if tensor.buffer is not None:
            return
        key = tensor.checkpoint_key
        assert key is not None
        cached = self._weight_cache.get(key)
        if cached is None:
            ckpt = self._checkpoint(tensor)
            if key not in ckpt.tensors:
                raise KeyError(f"{tensor.name}: checkpoint key {key!r} not in {ckpt.path}")
            host = ckpt.array(key)
            want = tuple(concrete_shape(tensor.spec))
            if tuple(host.shape) != want:
                raise ValueError(f"{tensor.name}: checkpoint {key} has physical shape {host.shape}, declared {want}")
            host_t = torch.from_numpy(np.array(host))
            want = TORCH_DTYPES[tensor.spec.dtype]
            if host_t.dtype != want:
                if host_t.element_size() != want.itemsize:
                    raise ValueError(f"{tensor.name}: checkpoint dtype {host_t.dtype} cannot back {tensor.spec.dtype}")
                host_t = host_t.view(want)
            with torch.cuda.stream(self.stream):
                cached = host_t.to(self.device)
            self._weight_cache[key] = cached
        with tensor.runtime_write_scope():
            tensor.buffer = cached

    # ------------------------------------------------------------- dispatch
    def dispatch(self, variant: ShaderVariant, **arguments: object) -> None:
        self._require_open()
        if not self._frame_stack:
            raise RuntimeError("RuntimeSession.dispatch requires an active rt.frame(...)")
        frame = self._frame_stack[-1]
        contract = variant.contract
        expected = {f.name for f in contract.fields}
        push_inputs = set()
        if contract.push_constants is not None:
            push_inputs = {f.value.name for f in contract.push_constants.fields if isinstance(f.value, PushConstantInput)}
        provided = set(arguments)
        if missing := expected - provided:
            raise ValueError(f"{variant.name} missing tensor fields: {sorted(missing)}")
        if missing_push := push_inputs - provided:
            raise ValueError(f"{variant.name} missing push constant inputs: {sorted(missing_push)}")
        if extra := provided - expected - push_inputs:
            raise ValueError(f"{variant.name} got unexpected fields: {sorted(extra)}")
        tensors: dict[str, LogicalTensor] = {}
        for f in contract.fields:
            arg = arguments[f.name]
            if not isinstance(arg, LogicalTensor):
                raise TypeError(f"{variant.name}.{f.name} expects LogicalTensor, got {type(arg).__name__}")
            arg.validate_declaration()
            tensors[f.name] = arg
        frame.used_tensors.extend(tensors.values())
        symbols = self._bind_shape_symbols(contract.fields, tensors)
        for f in contract.input_fields:
            self._materialize_read(tensors[f.name])
        for f in contract.output_fields:
            self._materialize_write(tensors[f.name], f.io_kind)
        push_values: dict[str, int | float] = {}
        if contract.push_constants is not None:
            for pc in contract.push_constants.fields:
                push_values[pc.name] = self._push_value(pc.value, tensors, symbols, arguments)
        dispatch_size = tuple(eval_expr(d, symbols) for d in contract.dispatch)
        if any(d == 0 for d in dispatch_size):
            for f in contract.output_fields:
                if tensor_nbytes(tensors[f.name].spec) != 0:
                    raise ValueError(f"{variant.name} resolved zero dispatch {dispatch_size} for a non-empty output")
            return
        op = self._ops.get(contract.class_name)
        if op is None:
            raise NotImplementedError(f"{variant.name}: no CUDA op for contract class {contract.class_name}")
        buffers = {name: t.buffer for name, t in tensors.items()}
        self._launch(op, variant, buffers, symbols, push_values)
        log = getattr(self, "_replay_log", None)
        if log is None:
            self._replay_log = log = []
        log.append(ReplayDispatch(op=op, variant=variant, tensors=dict(tensors), symbols=dict(symbols),
                                  push_values=dict(push_values), push_inputs=push_inputs_of(contract)))
        index = len(self._dispatch_records)
        self._dispatch_records.append(DispatchRecord(
            index=index, frame=frame.frame, shader=variant.name,
            reads=tuple((f.name, tensors[f.name]) for f in contract.input_fields),
            writes=tuple((f.name, tensors[f.name]) for f in contract.output_fields),
            symbols=tuple(sorted(symbols.items())), dispatch_size=dispatch_size,
            push_constant_values=tuple(sorted(push_values.items()))))
        for f in contract.output_fields:
            t = tensors[f.name]
            with t.runtime_write_scope():
                t.version += 1
                t.writer = DispatchWriter(frame=frame.frame, shader=variant.name, dispatch_index=index)
            frame.written_tensors.append(t)

    def _launch(self, op, variant: ShaderVariant, buffers, symbols, push_values) -> None:
        with torch.cuda.stream(self.stream):
            op(self, variant, buffers, symbols, push_values)

    def _push_value(self, value, tensors, symbols, arguments) -> int | float:
        if isinstance(value, PushConstantInput):
            v = arguments[value.name]
            return v if isinstance(v, int | float) else int(v)
        if isinstance(value, int | float) and not isinstance(value, bool):
            return value
        if callable(value):
            return value(tensors, symbols)
        return eval_expr(value, symbols)

    def _bind_shape_symbols(self, fields: tuple[TensorFieldSpec, ...], tensors: Mapping[str, LogicalTensor]) -> dict[str, int]:
        symbols: dict[str, int] = {}
        dtype_by_field: dict[str, str] = {}
        for f in fields:
            tensor, contract = tensors[f.name], f.contract
            dtype = contract.dtype
            if isinstance(dtype, DTypeReference):
                if dtype.field_name not in dtype_by_field:
                    raise ValueError(f"{f.name} references unknown dtype field {dtype.field_name}")
                allowed = (dtype_by_field[dtype.field_name],)
            elif isinstance(dtype, tuple):
                allowed = dtype
            else:
                allowed = (dtype,)
            if tensor.spec.dtype not in allowed:
                raise ValueError(f"{f.name} expects dtype {allowed}, got {tensor.spec.dtype} from {tensor.name}")
            dtype_by_field[f.name] = tensor.spec.dtype
            if len(tensor.spec.shape) != len(contract.shape):
                raise ValueError(f"{f.name} expects rank {len(contract.shape)}, got {len(tensor.spec.shape)} from {tensor.name}")
            for want, got in zip(contract.shape, tensor.spec.shape, strict=True):
                if not isinstance(got, int):
                    raise ValueError(f"{tensor.name} has unresolved shape {tensor.spec.shape}")
                if isinstance(want, int):
                    if got != want:
                        raise ValueError(f"{f.name} expects dim {want}, got {got}")
                elif isinstance(want, str):
                    prev = symbols.setdefault(want, got)
                    if prev != got:
                        raise ValueError(f"Shape symbol {want} bound to both {prev} and {got}")
                elif eval_expr(want, symbols) != got:
                    raise ValueError(f"{f.name} expects dim {eval_expr(want, symbols)}, got {got}")
            bind_tensor_layout_symbols(contract.layout, tensor.layout, symbols)
        return symbols

    # ------------------------------------------------------ materialization
    def _alloc(self, tensor: LogicalTensor) -> torch.Tensor:
        """Device storage for one tensor, allocated on the session stream so that the caching
        allocator orders its reuse after this stream's pending kernels."""
        with torch.cuda.stream(self.stream):
            return torch.empty(concrete_shape(tensor.spec), dtype=TORCH_DTYPES[tensor.spec.dtype], device=self.device)

    def _upload(self, tensor: LogicalTensor, value: object) -> None:
        arr = value.detach().cpu().numpy() if isinstance(value, torch.Tensor) else np.asarray(value)
        want = TORCH_DTYPES[tensor.spec.dtype]
        shape = concrete_shape(tensor.spec)
        host = torch.from_numpy(np.ascontiguousarray(arr))
        if host.numel() != int(np.prod(shape)):
            raise ValueError(f"{tensor.name}: value has {host.numel()} elements, declared shape {shape}")
        if host.dtype != want:
            same_kind = host.dtype.is_floating_point == want.is_floating_point
            host = host.view(want) if host.element_size() == want.itemsize and not same_kind else host.to(want)
        with torch.cuda.stream(self.stream):
            buf = host.reshape(shape).to(self.device)
        with tensor.runtime_write_scope():
            tensor.buffer = buf

    def _alias_view(self, tensor: LogicalTensor) -> None:
        source = tensor.alias_source
        assert source is not None
        if source.buffer is None:
            raise RuntimeError(f"{tensor.name} alias source {source.name} is not materialized")
        nbytes = tensor.alias_nbytes or tensor_nbytes(tensor.spec)
        raw = source.buffer.reshape(-1).view(torch.uint8)
        if tensor.alias_byte_offset + nbytes > raw.numel():
            raise RuntimeError(f"{tensor.name} alias range [{tensor.alias_byte_offset}, "
                               f"{tensor.alias_byte_offset + nbytes}) exceeds {source.name} size {raw.numel()}")
        view = raw[tensor.alias_byte_offset:tensor.alias_byte_offset + nbytes]
        view = view.view(TORCH_DTYPES[tensor.spec.dtype]).reshape(concrete_shape(tensor.spec))
        with tensor.runtime_write_scope():
            tensor.buffer = view
            tensor.version = source.version
            tensor.writer = source.writer

    def _materialize_read(self, tensor: LogicalTensor) -> None:
        if tensor.alias_source is not None:
            self._materialize_read(tensor.alias_source)
            self._alias_view(tensor)
            return
        if tensor.buffer is not None:
            return
        if tensor.role is TensorRole.WEIGHT:
            self._materialize_weight(tensor)
            return
        if tensor.memory is MemoryClass.SESSION_TENSOR:
            raise RuntimeError(f"{tensor.name} requires initialize_session_tensors(...) before use")
        if tensor.role is TensorRole.INPUT and tensor in self._inputs:
            self._upload(tensor, self._inputs[tensor])
            if tensor.lifetime in {TensorLifetime.FRAME, TensorLifetime.OP}:
                self._frame_tensors.append(tensor)
            return
        raise RuntimeError(f"{tensor.name} cannot be read before it is materialized or written")

    def _materialize_write(self, tensor: LogicalTensor, io_kind: IOKind) -> None:
        if tensor.alias_source is not None:
            raise RuntimeError(f"{tensor.name} is an alias of {tensor.alias_source.name} and cannot be written")
        if tensor.buffer is not None:
            return
        if io_kind is IOKind.INOUT:
            raise RuntimeError(f"{tensor.name} is read-write but was never initialized")
        with tensor.runtime_write_scope():
            tensor.buffer = self._alloc(tensor)
        if tensor.lifetime in {TensorLifetime.FRAME, TensorLifetime.OP}:
            self._frame_tensors.append(tensor)
        elif tensor.memory is MemoryClass.REQUEST_STATE or tensor.lifetime is TensorLifetime.REQUEST:
            self._request_tensors.add(tensor)

    def _drop(self, tensor: LogicalTensor) -> None:
        if tensor.buffer is None:
            return
        with tensor.runtime_write_scope():
            tensor.buffer = None
            tensor.writer = None

    def _release_frame_tensors(self) -> None:
        for t in self._frame_tensors:
            self._drop(t)
        self._frame_tensors = []

    def release_layer_workspace(self, layer_tensors: object, *, layer: str,
                                keep: Sequence[LogicalTensor] = ()) -> None:
        """Frees the frame-workspace activations of one layer before frame exit, except `keep` and the
        tensors they alias (src/torch2vk/runtime/materialization.py:423-448)."""
        self._require_open()
        if not layer:
            raise ValueError("release_layer_workspace requires a non-empty layer")
        keep_ids = set()
        for t in keep:
            while t is not None:
                keep_ids.add(id(t))
                t = t.alias_source
        for tensor in collect_named_logical_tensors(layer_tensors).values():
            if id(tensor) in keep_ids or tensor.layer != layer or tensor.buffer is None:
                continue
            if tensor.role is not TensorRole.ACTIVATION or tensor.memory is not MemoryClass.FRAME_WORKSPACE:
                continue
            if tensor.lifetime is not TensorLifetime.FRAME:
                continue
            self._drop(tensor)

    def release_frame_workspace(self, tensor: LogicalTensor) -> None:
        """Frees a frame / op-scratch tensor (through its alias chain) before frame exit; other
        tensors are left alone (src/torch2vk/runtime/materialization.py:451-461)."""
        self._require_open()
        while tensor.alias_source is not None:
            tensor = tensor.alias_source
        if tensor.memory not in {MemoryClass.FRAME_WORKSPACE, MemoryClass.OP_SCRATCH}:
            return
        if tensor.lifetime not in {TensorLifetime.FRAME, TensorLifetime.OP}:
            return
        self._drop(tensor)

    # -------------------------------------------------------------- readback
    def bind_model_tensors(self, model_tensors: object) -> None:
        """Binds (or replaces) the declared model tensors of this session
        (src/torch2vk/runtime/session.py:269-278)."""
        self._require_open()
        collect_named_logical_tensors(model_tensors)
        self._model_tensors = model_tensors

    # ------------------------------------------------------------- replay plans
    def build_replay_plan(self, *, name: str, frame: str,
                          readback_tensors: Mapping[str, LogicalTensor] | None = None) -> ReplayPlan:
        """A replayable copy of a finished frame's dispatches (src/torch2vk/runtime/session.py:381-393)."""
        self._require_open()
        return build_replay_plan_impl(self, name=name, frame=frame, readback_tensors=readback_tensors)

    def rebind_replay_plan(self, plan: ReplayPlan) -> None:
        rebind_replay_plan_impl(self, plan)

    def replay_plan_compatible(self, plan: ReplayPlan) -> bool:
        return replay_plan_compatible_impl(self, plan)

    def cached_replay_plans(self, namespace: str) -> tuple[ReplayPlan, ...]:
        """This session's live plans of the namespace, plus the plans instantiated from the
        namespace's on-disk templates (written by any earlier session with an artifact_dir) that
        match this session's model (src/torch2vk/runtime/replay_cache.py:28-49)."""
        from torch2vk_b200.runtime import replay_cache

        self._require_open()
        cache = getattr(self, "_replay_cache", None)
        if cache is None:
            self._replay_cache = cache = {}
        plans = [p for p in cache.get(namespace, []) if not p._closed and self.replay_plan_compatible(p)]
        templates = replay_cache.load_templates(self, namespace)
        have = {replay_cache.template_of(p) for p in plans}
        for template in templates:
            if template in have:
                continue
            plan = replay_cache.instantiate(self, template)
            if plan is not None:
                plans.append(plan)
                have.add(template)
        cache[namespace] = plans
        if not plans and templates:
            raise RuntimeError(f"Replay cache {namespace!r} exists but is incompatible with current model tensors")
        return tuple(plans)

    def cache_replay_plan(self, namespace: str, plan: ReplayPlan) -> None:
        """Caches the plan for this session and, with an artifact_dir, as an on-disk template."""
        from torch2vk_b200.runtime import replay_cache

        self._require_open()
        if plan._closed:
            raise RuntimeError(f"Cannot cache closed ReplayPlan {plan.name!r}")
        if plan.session is not self:
            raise ValueError("ReplayPlan belongs to a different RuntimeSession")
        cache = getattr(self, "_replay_cache", None)
        if cache is None:
            self._replay_cache = cache = {}
        plans = cache.setdefault(namespace, [])
        if not any(p is plan for p in plans):
            plans.append(plan)
        replay_cache.store_template(self, namespace, plan)

    def synchronize(self) -> None:
        self.stream.synchronize()

    def readback(self, tensor: LogicalTensor) -> np.ndarray:
        self._require_open()
        self.synchronize()
        self._materialize_read(tensor)
        buf = tensor.buffer
        if buf is None:
            raise RuntimeError(f"{tensor.name} is not materialized")
        host = buf.detach().cpu()
        if host.dtype in (torch.uint16, torch.uint32):
            return host.view(torch.int16 if host.dtype == torch.uint16 else torch.int32).numpy().view(
                np.uint16 if host.dtype == torch.uint16 else np.uint32)
        return host.numpy()

    def read_request_state(self, tensor: LogicalTensor) -> np.ndarray:
        if tensor.memory is not MemoryClass.REQUEST_STATE:
            raise ValueError(f"{tensor.name} is not request state")
        return self.readback(tensor)

    # ---------------------------------------------------------------- close
    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        self.synchronize()
        for t in list(self._frame_tensors) + list(self._request_tensors):
            self._drop(t)
        if self._model_tensors is not None:
            for t in collect_named_logical_tensors(self._model_tensors).values():
                if t.memory in {MemoryClass.MODEL_WEIGHT, MemoryClass.SESSION_TENSOR}:
                    self._drop(t)
        self._weight_cache.clear()
        for ck in self._checkpoints.values():
            ck.close()
        self._checkpoints.clear()

    def _require_open(self) -> None:
        if self._closed:
            raise RuntimeError("RuntimeSession is closed")

    def _named_model_tensors(self) -> dict[str, LogicalTensor]:
        if self._model_tensors is None:
            raise RuntimeError("RuntimeSession.open(..., model_tensors=...) is required")
        return collect_named_logical_tensors(self._model_tensors)

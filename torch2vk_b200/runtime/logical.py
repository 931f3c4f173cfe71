"""Logical tensor declarations (src/torch2vk/runtime/logical.py:25-389, the binding rules of
docs/frame-and-logical-tensor.md) for the CUDA backend.

Model code declares LogicalTensors (spec, role, memory class, lifetime, GGUF
checkpoint_key); only the runtime writes their runtime state.  Here the
materialized `buffer` is a torch CUDA tensor owned by the RuntimeSession.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass, field, fields, is_dataclass
from enum import StrEnum
from typing import Literal

from torch2vk_b200.runtime.types import (CONTIGUOUS_LAYOUT, TensorLayout, TensorSpec, dtype_nbytes, tensor_nbytes,
                                         validate_tensor_layout)


class TensorRole(StrEnum):
    MISSING_VALUE = "missing_value"
    INPUT = "input"
    WEIGHT = "weight"
    ACTIVATION = "activation"
    SCRATCH = "scratch"
    OUTPUT = "output"
    STATE = "state"


class TensorSemantic(StrEnum):
    LOGITS = "logits"
    TOKEN = "token"
    KV_CACHE = "kv_cache"
    MASK = "mask"
    WAVEFORM = "waveform"


class MemoryClass(StrEnum):
    MISSING_VALUE = "missing_value"
    MODEL_WEIGHT = "model_weight"
    SESSION_TENSOR = "session_tensor"
    REQUEST_STATE = "request_state"
    FRAME_WORKSPACE = "frame_workspace"
    OP_SCRATCH = "op_scratch"
    HOST_INPUT = "host_input"
    HOST_OUTPUT = "host_output"


class TensorLifetime(StrEnum):
    MISSING_VALUE = "missing_value"
    MODEL = "model"
    REQUEST = "request"
    FRAME = "frame"
    OP = "op"
    EXTERNAL = "external"


_DEFAULTS = {
    TensorRole.WEIGHT: (MemoryClass.MODEL_WEIGHT, TensorLifetime.MODEL),
    TensorRole.INPUT: (MemoryClass.HOST_INPUT, TensorLifetime.FRAME),
    TensorRole.ACTIVATION: (MemoryClass.FRAME_WORKSPACE, TensorLifetime.FRAME),
    TensorRole.SCRATCH: (MemoryClass.OP_SCRATCH, TensorLifetime.OP),
    TensorRole.OUTPUT: (MemoryClass.HOST_OUTPUT, TensorLifetime.FRAME),
    TensorRole.STATE: (MemoryClass.REQUEST_STATE, TensorLifetime.REQUEST),
}


def default_memory_lifetime_for_role(role: TensorRole) -> tuple[MemoryClass, TensorLifetime] | None:
    return _DEFAULTS.get(role)


@dataclass(frozen=True, slots=True)
class ComparePolicy:
    kind: Literal["tensor", "token", "waveform"] = "tensor"
    rtol: float = 1e-4
    atol: float = 1e-4
    max_abs: float | None = None


@dataclass(frozen=True, slots=True)
class DispatchWriter:
    frame: str
    shader: str
    dispatch_index: int


_RUNTIME_FIELDS = ("buffer", "version", "writer")


@dataclass(slots=True, eq=False)
class LogicalTensor:
    spec: TensorSpec
    role: TensorRole
    memory: MemoryClass
    lifetime: TensorLifetime
    name: str = ""
    layout: TensorLayout = CONTIGUOUS_LAYOUT
    semantic: TensorSemantic | None = None
    checkpoint: str | None = None
    checkpoint_key: str | None = None
    reference_key: str | None = None
    layer: str | None = None
    _runtime_writable: bool = field(default=False, init=False, repr=False)
    _buffer: object | None = field(default=None, init=False, repr=False)
    _version: int = field(default=0, init=False, repr=False)
    _writer: DispatchWriter | None = field(default=None, init=False, repr=False)
    _alias_source: "LogicalTensor | None" = field(default=None, init=False, repr=False)
    _alias_byte_offset: int = field(default=0, init=False, repr=False)
    _alias_nbytes: int | None = field(default=None, init=False, repr=False)

    @contextmanager
    def runtime_write_scope(self) -> Iterator[None]:
        previous = self._runtime_writable
        self._runtime_writable = True
        try:
            yield
        finally:
            self._runtime_writable = previous

    def _require_runtime_writable(self, what: str) -> None:
        if not self._runtime_writable:
            raise RuntimeError(f"{self.name}.{what} is runtime state and cannot be written during declaration")

    @property
    def buffer(self) -> object | None:
        """The materialized torch CUDA tensor (runtime-owned), or None."""
        return self._buffer

    @buffer.setter
    def buffer(self, value: object | None) -> None:
        self._require_runtime_writable("buffer")
        self._buffer = value

    @property
    def version(self) -> int:
        return self._version

    @version.setter
    def version(self, value: int) -> None:
        self._require_runtime_writable("version")
        self._version = value

    @property
    def writer(self) -> DispatchWriter | None:
        return self._writer

    @writer.setter
    def writer(self, value: DispatchWriter | None) -> None:
        self._require_runtime_writable("writer")
        self._writer = value

    @property
    def alias_source(self) -> "LogicalTensor | None":
        """The tensor whose storage this one views (bind_logical_tensor_alias), or None."""
        return self._alias_source

    @alias_source.setter
    def alias_source(self, value: "LogicalTensor | None") -> None:
        self._require_runtime_writable("alias_source")
        self._alias_source = value
        if value is None:
            self._alias_byte_offset = 0
            self._alias_nbytes = None

    @property
    def alias_byte_offset(self) -> int:
        return self._alias_byte_offset

    @alias_byte_offset.setter
    def alias_byte_offset(self, value: int) -> None:
        self._require_runtime_writable("alias_byte_offset")
        if value < 0:
            raise ValueError(f"{self.name} alias byte offset must be non-negative, got {value}")
        self._alias_byte_offset = value

    @property
    def alias_nbytes(self) -> int | None:
        return self._alias_nbytes

    @alias_nbytes.setter
    def alias_nbytes(self, value: int | None) -> None:
        self._require_runtime_writable("alias_nbytes")
        if value is not None and value <= 0:
            raise ValueError(f"{self.name} alias nbytes must be positive, got {value}")
        self._alias_nbytes = value

    @property
    def concrete_shape(self) -> tuple[int, ...]:
        out = []
        for dim in self.spec.shape:
            if not isinstance(dim, int):
                raise ValueError(f"{self.name} has unresolved symbolic shape {self.spec.shape}")
            out.append(dim)
        return tuple(out)

    def fill_missing_declaration_defaults(self) -> None:
        defaults = default_memory_lifetime_for_role(self.role)
        if defaults is None:
            return
        if self.memory is MemoryClass.MISSING_VALUE:
            self.memory = defaults[0]
        if self.lifetime is TensorLifetime.MISSING_VALUE:
            self.lifetime = defaults[1]

    def validate_declaration(self) -> None:
        self.fill_missing_declaration_defaults()
        if not self.name or any(part == "" for part in self.name.split(".")):
            raise ValueError(f"LogicalTensor name is empty or has an empty component: {self.name!r}")
        if (self.role is TensorRole.MISSING_VALUE or self.memory is MemoryClass.MISSING_VALUE
                or self.lifetime is TensorLifetime.MISSING_VALUE or self.spec.dtype == "missing_value"):
            raise ValueError(f"{self.name} has unresolved missing LogicalTensor metadata")
        if self.role is TensorRole.WEIGHT and not self.checkpoint_key:
            raise ValueError(f"{self.name} is a weight tensor but checkpoint_key is not set")
        dtype_nbytes(self.spec.dtype)
        if not self.spec.shape:
            raise ValueError(f"{self.name} shape must have fixed rank")
        validate_tensor_layout(self.layout, self.spec.shape)
        _validate_role_memory_lifetime(self)


def _validate_role_memory_lifetime(t: LogicalTensor) -> None:
    role, memory, lifetime = t.role, t.memory, t.lifetime
    if role is TensorRole.ACTIVATION and (memory is not MemoryClass.FRAME_WORKSPACE or lifetime is not TensorLifetime.FRAME):
        raise ValueError(f"{t.name} activation must use FRAME_WORKSPACE/FRAME")
    if role is TensorRole.SCRATCH and (memory is not MemoryClass.OP_SCRATCH or lifetime is not TensorLifetime.OP):
        raise ValueError(f"{t.name} scratch must use OP_SCRATCH/OP")
    if role is TensorRole.STATE and (memory is not MemoryClass.REQUEST_STATE or lifetime is not TensorLifetime.REQUEST):
        raise ValueError(f"{t.name} state must use REQUEST_STATE/REQUEST")
    if role is TensorRole.WEIGHT and (memory is not MemoryClass.MODEL_WEIGHT or lifetime is not TensorLifetime.MODEL):
        raise ValueError(f"{t.name} weight must use MODEL_WEIGHT/MODEL")
    if role is TensorRole.OUTPUT:
        if memory not in {MemoryClass.FRAME_WORKSPACE, MemoryClass.HOST_OUTPUT, MemoryClass.REQUEST_STATE}:
            raise ValueError(f"{t.name} output cannot use memory={memory}")
        if lifetime not in {TensorLifetime.FRAME, TensorLifetime.REQUEST}:
            raise ValueError(f"{t.name} output cannot use lifetime={lifetime}")
    if role is TensorRole.INPUT:
        if memory is MemoryClass.SESSION_TENSOR:
            if lifetime is not TensorLifetime.MODEL:
                raise ValueError(f"{t.name} session tensor input must use MODEL lifetime")
            return
        if memory not in {MemoryClass.HOST_INPUT, MemoryClass.REQUEST_STATE}:
            raise ValueError(f"{t.name} input cannot use memory={memory}")
        if lifetime not in {TensorLifetime.FRAME, TensorLifetime.REQUEST}:
            raise ValueError(f"{t.name} input cannot use lifetime={lifetime}")


def bind_logical_tensor_alias(src: LogicalTensor, dst: LogicalTensor, *, byte_offset: int = 0,
                              nbytes: int | None = None) -> None:
    """dst views src's storage at byte_offset (src/torch2vk/runtime/logical.py:284-316, same checks)."""
    src.validate_declaration()
    dst.validate_declaration()
    src_nbytes, dst_nbytes = tensor_nbytes(src.spec), tensor_nbytes(dst.spec)
    if nbytes is None and byte_offset == 0 and src_nbytes != dst_nbytes:
        raise ValueError(f"{dst.name} cannot alias {src.name}: byte size differs ({dst_nbytes} != {src_nbytes})")
    view_nbytes = dst_nbytes if nbytes is None else nbytes
    if view_nbytes != dst_nbytes:
        raise ValueError(f"{dst.name} cannot alias {src.name}: view byte size differs from dst "
                         f"({view_nbytes} != {dst_nbytes})")
    if byte_offset < 0:
        raise ValueError(f"{dst.name} cannot alias {src.name}: byte_offset must be non-negative")
    if byte_offset + view_nbytes > src_nbytes:
        raise ValueError(f"{dst.name} cannot alias {src.name}: byte range [{byte_offset}, {byte_offset + view_nbytes}) "
                         f"exceeds source size {src_nbytes}")
    with dst.runtime_write_scope():
        dst.alias_source = src
        dst.alias_byte_offset = byte_offset
        dst.alias_nbytes = view_nbytes


def bind_logical_tensor_names(root: object, prefix: str = "", *, overwrite: bool = True) -> None:
    seen: set[int] = set()

    def bind(value: object, path: str) -> None:
        if isinstance(value, LogicalTensor):
            if id(value) in seen:
                return
            seen.add(id(value))
            if not overwrite and value.name:
                return
            if not path:
                raise ValueError("LogicalTensor root cannot be named from an empty path")
            value.name = path
            return
        if is_dataclass(value) and not isinstance(value, type):
            for f in fields(value):
                bind(getattr(value, f.name), f.name if not path else f"{path}.{f.name}")
        elif isinstance(value, tuple | list):
            for i, item in enumerate(value):
                bind(item, str(i) if not path else f"{path}.{i}")

    bind(root, prefix)


def collect_named_logical_tensors(root: object) -> dict[str, LogicalTensor]:
    out: dict[str, LogicalTensor] = {}
    seen: set[int] = set()

    def collect(value: object) -> None:
        if isinstance(value, LogicalTensor):
            if id(value) in seen:
                return
            seen.add(id(value))
            if not value.name:
                raise ValueError("LogicalTensor name must be non-empty")
            existing = out.get(value.name)
            if existing is not None and existing is not value:
                raise RuntimeError(f"Model tensors contain multiple LogicalTensor objects named {value.name!r}")
            out[value.name] = value
        elif is_dataclass(value) and not isinstance(value, type):
            for f in fields(value):
                collect(getattr(value, f.name))
        elif isinstance(value, tuple | list):
            for item in value:
                collect(item)

    collect(root)
    return out

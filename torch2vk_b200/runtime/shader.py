"""Shader contracts and variants: the declaration types of torch2vk.runtime.shader
(src/torch2vk/runtime/shader.py:17-341) for the CUDA backend.

A ShaderVariant still names an op (`name`, `family`) and carries its
ShaderContract (class_name, fields with dtype / symbolic shape / layout, push
constants, dispatch grid).  Here `source` names the sm_100a op that serves
the contract instead of holding GLSL; RuntimeSession.dispatch looks the op up
by `contract.class_name` in the CUDA op table.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping
from dataclasses import dataclass, field as dataclass_field
from enum import StrEnum
from typing import TYPE_CHECKING, TypeAlias

from torch2vk_b200.runtime.types import CONTIGUOUS_LAYOUT, Dim, TensorLayout

if TYPE_CHECKING:
    from torch2vk_b200.runtime.logical import LogicalTensor


@dataclass(frozen=True, slots=True)
class CeilDivExpr:
    lhs: "ExprDim"
    rhs: "ExprDim"


@dataclass(frozen=True, slots=True)
class MulExpr:
    lhs: "ExprDim"
    rhs: "ExprDim"


@dataclass(frozen=True, slots=True)
class AddExpr:
    lhs: "ExprDim"
    rhs: "ExprDim"


ExprDim: TypeAlias = Dim | CeilDivExpr | MulExpr | AddExpr


def ceil_div(lhs: ExprDim, rhs: ExprDim) -> CeilDivExpr:
    return CeilDivExpr(lhs=lhs, rhs=rhs)


def mul(lhs: ExprDim, rhs: ExprDim) -> MulExpr:
    return MulExpr(lhs=lhs, rhs=rhs)


def add(lhs: ExprDim, rhs: ExprDim) -> AddExpr:
    return AddExpr(lhs=lhs, rhs=rhs)


class DescriptorType(StrEnum):
    STORAGE_BUFFER = "storage_buffer"


class IOKind(StrEnum):
    INPUT = "input"
    OUTPUT = "output"
    INOUT = "inout"


class PushConstantType(StrEnum):
    UINT32 = "uint32"
    INT32 = "int32"
    FLOAT32 = "float32"
    UINT64 = "uint64"


@dataclass(frozen=True, slots=True)
class DTypeReference:
    field_name: str


def same_as(field_name: str) -> DTypeReference:
    return DTypeReference(field_name=field_name)


@dataclass(frozen=True, slots=True)
class TensorContract:
    dtype: str | tuple[str, ...] | DTypeReference
    shape: tuple[ExprDim, ...]
    layout: TensorLayout = CONTIGUOUS_LAYOUT


@dataclass(frozen=True, slots=True)
class TensorFieldSpec:
    name: str
    io_kind: IOKind
    role: str
    contract: TensorContract
    descriptor_type: DescriptorType = DescriptorType.STORAGE_BUFFER


@dataclass(frozen=True, slots=True)
class PushConstantInput:
    name: str


PushConstantResolver: TypeAlias = Callable[[Mapping[str, object], Mapping[str, int]], int | float]
PushConstantValue: TypeAlias = ExprDim | PushConstantInput | PushConstantResolver | int | float


@dataclass(frozen=True, slots=True)
class PushConstantFieldSpec:
    name: str
    dtype: PushConstantType
    offset: int
    value: PushConstantValue
    dynamic: bool = False

    @property
    def size(self) -> int:
        return 8 if self.dtype is PushConstantType.UINT64 else 4


@dataclass(frozen=True, slots=True)
class PushConstantSpec:
    size: int
    fields: tuple[PushConstantFieldSpec, ...]


@dataclass(frozen=True, slots=True)
class ParamsBufferFieldSpec:
    name: str
    dtype: PushConstantType
    offset: int
    value: PushConstantValue

    @property
    def size(self) -> int:
        return 8 if self.dtype is PushConstantType.UINT64 else 4


@dataclass(frozen=True, slots=True)
class ParamsBufferSpec:
    size: int
    fields: tuple[ParamsBufferFieldSpec, ...]
    binding_index: int


@dataclass(frozen=True, slots=True)
class ShaderContract:
    class_name: str
    shader_name: str
    fields: tuple[TensorFieldSpec, ...]
    dispatch: tuple[ExprDim, ExprDim, ExprDim]
    push_constants: PushConstantSpec | None = None
    params_buffer: ParamsBufferSpec | None = None

    @property
    def input_fields(self) -> tuple[TensorFieldSpec, ...]:
        return tuple(f for f in self.fields if f.io_kind in (IOKind.INPUT, IOKind.INOUT))

    @property
    def output_fields(self) -> tuple[TensorFieldSpec, ...]:
        return tuple(f for f in self.fields if f.io_kind in (IOKind.OUTPUT, IOKind.INOUT))

    def validate_definition(self) -> None:
        if not self.class_name or not self.shader_name:
            raise ValueError("ShaderContract class_name and shader_name must be non-empty")
        if len(self.dispatch) != 3:
            raise ValueError(f"{self.shader_name} dispatch must be rank 3")
        names: set[str] = set()
        for f in self.fields:
            if not f.name or f.name in names:
                raise ValueError(f"{self.shader_name} has an empty or duplicate field {f.name!r}")
            names.add(f.name)
        if self.push_constants is not None:
            seen: set[str] = set()
            occupied: set[int] = set()
            for pc in self.push_constants.fields:
                if pc.name in seen:
                    raise ValueError(f"{self.shader_name} duplicate push constant field {pc.name}")
                seen.add(pc.name)
                if pc.offset < 0 or pc.offset + pc.size > self.push_constants.size:
                    raise ValueError(f"{self.shader_name}.{pc.name} push constant range is out of bounds")
                span = set(range(pc.offset, pc.offset + pc.size))
                if span & occupied:
                    raise ValueError(f"{self.shader_name}.{pc.name} overlaps another push constant")
                occupied |= span


@dataclass(frozen=True, slots=True)
class ShaderVariant:
    """An op declaration.  The reference's GLSL-related fields (source text, SPIR-V path,
    specialization constants, include dirs, defines, execution requirements) are accepted
    so generated shader modules construct unchanged; dispatch uses only `contract`."""

    name: str
    family: str
    contract: ShaderContract
    source: str = "cuda"
    precompiled_spv_path: object | None = None
    specialization_constants: tuple[tuple[int, int], ...] | None = None
    include_dirs: tuple[object, ...] = ()
    compile_defines: tuple[str, ...] = ()
    execution_requirements: object | None = None

    def __post_init__(self) -> None:
        if self.name != self.contract.shader_name:
            raise ValueError(f"ShaderVariant name {self.name!r} must equal contract shader_name")
        if not self.family:
            raise ValueError(f"{self.name} family must be non-empty")
        self.contract.validate_definition()

    def __call__(self, rt: object, **arguments: object) -> None:
        getattr(rt, "dispatch")(self, **arguments)


def collect_shader_variants(source: object) -> dict[str, ShaderVariant]:
    return {v.name: v for v in (getattr(source, a) for a in dir(source)) if isinstance(v, ShaderVariant)}


@dataclass(frozen=True, slots=True)
class DispatchRecord:
    index: int
    frame: str
    shader: str
    reads: tuple[tuple[str, "LogicalTensor"], ...]
    writes: tuple[tuple[str, "LogicalTensor"], ...]
    symbols: tuple[tuple[str, int], ...]
    dispatch_size: tuple[int, int, int]
    push_constant_values: tuple[tuple[str, int | float], ...] = dataclass_field(default_factory=tuple)


def referenced_symbols(expr: ExprDim) -> tuple[str, ...]:
    if isinstance(expr, str):
        return (expr,)
    if isinstance(expr, int):
        return ()
    if isinstance(expr, CeilDivExpr | MulExpr | AddExpr):
        return referenced_symbols(expr.lhs) + referenced_symbols(expr.rhs)
    raise TypeError(f"Unsupported expression dim {expr!r}")


def eval_expr(expr: ExprDim, symbols: Mapping[str, int]) -> int:
    if isinstance(expr, int):
        return int(expr)
    if isinstance(expr, str):
        try:
            return int(symbols[expr])
        except KeyError as exc:
            raise ValueError(f"Unresolved shape symbol {expr!r}") from exc
    if isinstance(expr, CeilDivExpr):
        rhs = eval_expr(expr.rhs, symbols)
        if rhs <= 0:
            raise ValueError(f"ceil_div rhs must be positive, got {rhs}")
        return (eval_expr(expr.lhs, symbols) + rhs - 1) // rhs
    if isinstance(expr, MulExpr):
        return eval_expr(expr.lhs, symbols) * eval_expr(expr.rhs, symbols)
    if isinstance(expr, AddExpr):
        return eval_expr(expr.lhs, symbols) + eval_expr(expr.rhs, symbols)
    raise TypeError(f"Unsupported expression dim {expr!r}")

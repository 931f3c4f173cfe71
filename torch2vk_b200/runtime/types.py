"""Tensor metadata types: the names generated torch2vk model code imports from
torch2vk.vulkan.types (src/torch2vk/vulkan/types.py:14-310), restated for the CUDA backend.

TensorSpec, the layout dataclasses (contiguous, strided, GGUF block layouts
Q4_K words / Q6_K halfwords / Q8_0 halfwords) and their constructor functions
keep the reference's names and fields so model declarations bind unchanged.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from enum import StrEnum
from typing import TypeAlias

Dim: TypeAlias = int | str
TensorShape: TypeAlias = tuple[Dim, ...]


class Residency(StrEnum):
    DEVICE = "device"
    HOST = "host"


@dataclass(frozen=True, slots=True)
class ContiguousLayout:
    kind: str = "contiguous"


@dataclass(frozen=True, slots=True)
class AnyStridedLayout:
    kind: str = "any_strided"


@dataclass(frozen=True, slots=True)
class StridedLayout:
    strides: tuple[Dim, ...]
    kind: str = "strided"


@dataclass(frozen=True, slots=True)
class Q4KWordsLayout:
    logical_k: Dim
    block_size: int = 256
    words_per_block: int = 36


@dataclass(frozen=True, slots=True)
class Q8_0HalfwordsLayout:
    logical_k: Dim
    block_size: int = 32
    halfwords_per_block: int = 17


@dataclass(frozen=True, slots=True)
class Q6KHalfwordsLayout:
    logical_k: Dim
    block_size: int = 256
    halfwords_per_block: int = 105


TensorLayout: TypeAlias = ContiguousLayout | AnyStridedLayout | StridedLayout | Q4KWordsLayout | Q8_0HalfwordsLayout | Q6KHalfwordsLayout

CONTIGUOUS_LAYOUT = ContiguousLayout()
ANY_STRIDED_LAYOUT = AnyStridedLayout()


def strided_layout(*strides: Dim) -> StridedLayout:
    return StridedLayout(strides=tuple(strides))


def q4_k_words_layout(*, logical_k: Dim, block_size: int = 256, words_per_block: int = 36) -> Q4KWordsLayout:
    return Q4KWordsLayout(logical_k=logical_k, block_size=block_size, words_per_block=words_per_block)


def q8_0_halfwords_layout(*, logical_k: Dim, block_size: int = 32, halfwords_per_block: int = 17) -> Q8_0HalfwordsLayout:
    return Q8_0HalfwordsLayout(logical_k=logical_k, block_size=block_size, halfwords_per_block=halfwords_per_block)


def q6_k_halfwords_layout(*, logical_k: Dim, block_size: int = 256, halfwords_per_block: int = 105) -> Q6KHalfwordsLayout:
    return Q6KHalfwordsLayout(logical_k=logical_k, block_size=block_size, halfwords_per_block=halfwords_per_block)


@dataclass(frozen=True, slots=True)
class TensorSpec:
    dtype: str
    shape: TensorShape
    residency: Residency = Residency.DEVICE

    @property
    def ndim(self) -> int:
        return len(self.shape)

    def with_shape(self, *shape: Dim) -> "TensorSpec":
        return TensorSpec(dtype=self.dtype, shape=shape, residency=self.residency)


_DTYPE_NBYTES = {"bool": 4, "float32": 4, "float64": 8, "float16": 2, "bfloat16": 2, "int8": 1, "uint8": 1,
                 "int16": 2, "uint16": 2, "int32": 4, "uint32": 4, "int64": 8}


def dtype_nbytes(dtype: str) -> int:
    try:
        return _DTYPE_NBYTES[dtype]
    except KeyError as exc:
        raise ValueError(f"Unsupported tensor dtype: {dtype}") from exc


def concrete_shape(spec: TensorSpec) -> tuple[int, ...]:
    out = []
    for dim in spec.shape:
        if not isinstance(dim, int):
            raise ValueError(f"Expected concrete tensor shape, got {spec.shape}")
        out.append(dim)
    return tuple(out)


def tensor_nbytes(spec: TensorSpec) -> int:
    n = 1
    for d in concrete_shape(spec):
        n *= d
    return n * dtype_nbytes(spec.dtype)


def validate_tensor_layout(layout: TensorLayout, shape: TensorShape) -> None:
    if isinstance(layout, StridedLayout) and len(layout.strides) != len(shape):
        raise ValueError(f"strided layout rank {len(layout.strides)} != tensor rank {len(shape)}")


def _resolve(dim: Dim, symbols: Mapping[str, int] | None) -> Dim:
    if isinstance(dim, str) and symbols is not None and dim in symbols:
        return symbols[dim]
    return dim


def bind_tensor_layout_symbols(expected: TensorLayout, actual: TensorLayout, symbols: dict[str, int]) -> None:
    """Binds logical_k (and strides) symbols of a contract layout against a tensor's layout."""
    if isinstance(expected, AnyStridedLayout):
        if not isinstance(actual, ContiguousLayout | StridedLayout):
            raise ValueError(f"expected a strided or contiguous layout, got {actual}")
        return
    if type(expected) is not type(actual):
        raise ValueError(f"layout {type(actual).__name__} does not match contract {type(expected).__name__}")
    pairs: list[tuple[Dim, Dim]] = []
    if isinstance(expected, StridedLayout):
        pairs = list(zip(expected.strides, actual.strides, strict=True))
    elif isinstance(expected, Q4KWordsLayout | Q6KHalfwordsLayout | Q8_0HalfwordsLayout):
        pairs = [(expected.logical_k, actual.logical_k)]
    for want, got in pairs:
        got = _resolve(got, symbols)
        if isinstance(want, str):
            if not isinstance(got, int):
                raise ValueError(f"layout symbol {want} bound to unresolved {got}")
            prev = symbols.setdefault(want, got)
            if prev != got:
                raise ValueError(f"Shape symbol {want} bound to both {prev} and {got}")
        elif want != got:
            raise ValueError(f"layout expects {want}, got {got}")

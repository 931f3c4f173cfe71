"""RoPE cos/sin tables (src/torch2vk/runtime/rope_table.py:22-190): the same declarations
and helper, served by the sm_100a rope_table kernel through the CUDA op table."""

from __future__ import annotations

from dataclasses import dataclass

from torch2vk_b200.runtime.logical import LogicalTensor, MemoryClass, TensorLifetime, TensorRole
from torch2vk_b200.runtime.types import TensorSpec
from torch2vk_b200.runtime.variants import ROPE_TABLE_F32


@dataclass(frozen=True, slots=True)
class RopeTableTensors:
    cos: LogicalTensor
    sin: LogicalTensor


def run_rope_table_f32(rt, *, start_position: int, theta: float, cos: LogicalTensor, sin: LogicalTensor,
                       frame_name: str) -> None:
    if cos.spec.dtype != "float16":
        raise ValueError(f"unsupported RoPE table dtype on the CUDA backend: {cos.spec.dtype}")
    with rt.frame(frame_name):
        ROPE_TABLE_F32(rt, start_position=start_position, theta=theta, cos=cos, sin=sin)


def _declare(name: str, *, batch: int, sequence_length: int, head_dim: int, dtype: str) -> LogicalTensor:
    return LogicalTensor(name=name, spec=TensorSpec(dtype=dtype, shape=(batch, sequence_length, head_dim)),
                         role=TensorRole.STATE, memory=MemoryClass.REQUEST_STATE, lifetime=TensorLifetime.REQUEST)


def declare_rope_table_tensors(prefix: str, *, batch: int, sequence_length: int, head_dim: int,
                               dtype: str = "float16") -> RopeTableTensors:
    kw = dict(batch=batch, sequence_length=sequence_length, head_dim=head_dim, dtype=dtype)
    return RopeTableTensors(cos=_declare(f"{prefix}.cos", **kw), sin=_declare(f"{prefix}.sin", **kw))

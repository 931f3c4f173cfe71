"""Execution-requirement declarations attached to reference shader variants
(src/torch2vk/vulkan/shader_execution_requirements.py:22-60).  They describe
Vulkan subgroup / cooperative-matrix / storage features; the CUDA backend
accepts and keeps them so that generated shader modules import unchanged,
and ignores them at dispatch."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True, slots=True)
class SubgroupRequirements:
    required_size: int
    require_full_subgroups: bool = False


@dataclass(frozen=True, slots=True)
class CooperativeMatrixRequirements:
    scope: str
    m_size: int
    n_size: int
    k_size: int
    a_type: str
    b_type: str
    c_type: str
    result_type: str
    saturating_accumulation: bool = False


@dataclass(frozen=True, slots=True)
class ShaderExecutionRequirements:
    subgroup: SubgroupRequirements | None = None
    cooperative_matrix: CooperativeMatrixRequirements | None = None
    require_integer_dot_product: bool = False
    require_shader_int64: bool = False
    require_buffer_device_address: bool = False
    require_storage_buffer_16bit_access: bool = False

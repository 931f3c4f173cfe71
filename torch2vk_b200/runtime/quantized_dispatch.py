"""run_quantized_linear: picks the Q4_K / Q6_K / Q8_0 variant by the weight's layout
(src/torch2vk/runtime/quantized_dispatch.py:15-35), same signature and errors."""

from __future__ import annotations

from typing import TYPE_CHECKING

from torch2vk_b200.runtime.logical import LogicalTensor
from torch2vk_b200.runtime.shader import ShaderVariant
from torch2vk_b200.runtime.types import Q4KWordsLayout, Q6KHalfwordsLayout, Q8_0HalfwordsLayout

if TYPE_CHECKING:
    from torch2vk_b200.runtime.session import RuntimeSession


def run_quantized_linear(rt: "RuntimeSession", *, q4: ShaderVariant, q6: ShaderVariant, q8: ShaderVariant,
                         x: LogicalTensor, weight: LogicalTensor, output: LogicalTensor) -> None:
    if isinstance(weight.layout, Q6KHalfwordsLayout):
        q6(rt, x=x, weight=weight, output=output)
    elif isinstance(weight.layout, Q8_0HalfwordsLayout):
        q8(rt, x=x, weight=weight, output=output)
    elif isinstance(weight.layout, Q4KWordsLayout):
        q4(rt, x=x, weight=weight, output=output)
    else:
        raise ValueError(f"{weight.name} expected Q4_K, Q6_K, or Q8_0 layout, got {weight.layout}")

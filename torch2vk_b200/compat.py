"""Drop-in module aliases: `import torch2vk.runtime.session` (and the other modules
generated torch2vk model code imports) resolve to this package's CUDA backend.

install() registers, in sys.modules,
  torch2vk.runtime.shader          -> torch2vk_b200.runtime.shader
  torch2vk.runtime.logical         -> torch2vk_b200.runtime.logical
  torch2vk.runtime.session         -> torch2vk_b200.runtime.session
  torch2vk.runtime.quantized_dispatch -> torch2vk_b200.runtime.quantized_dispatch
  torch2vk.runtime.rope_table      -> torch2vk_b200.runtime.rope_table
  torch2vk.runtime.replay          -> torch2vk_b200.runtime.replay
  torch2vk.runtime.replay_cache_key -> torch2vk_b200.runtime.replay_cache_key
  torch2vk.vulkan.types            -> torch2vk_b200.runtime.types
  torch2vk.vulkan.shader_execution_requirements -> torch2vk_b200.runtime.execution_requirements
  torch2vk.quantize                -> torch2vk_b200.quantize
so that a model package generated for the reference (its shaders/, tensors/
and dispatch/ modules) runs unchanged: each ShaderVariant it builds is this
package's ShaderVariant, and `VARIANT(rt, **fields)` reaches
RuntimeSession.dispatch, which launches the sm_100a kernels named by the
CUDA op table.  Only the modules listed are provided.
"""

from __future__ import annotations

import importlib
import sys
import types

ALIASES = {
    "torch2vk.runtime.shader": "torch2vk_b200.runtime.shader",
    "torch2vk.runtime.logical": "torch2vk_b200.runtime.logical",
    "torch2vk.runtime.session": "torch2vk_b200.runtime.session",
    "torch2vk.runtime.quantized_dispatch": "torch2vk_b200.runtime.quantized_dispatch",
    "torch2vk.runtime.rope_table": "torch2vk_b200.runtime.rope_table",
    "torch2vk.runtime.replay": "torch2vk_b200.runtime.replay",
    "torch2vk.runtime.replay_cache_key": "torch2vk_b200.runtime.replay_cache_key",
    "torch2vk.vulkan.types": "torch2vk_b200.runtime.types",
    "torch2vk.vulkan.shader_execution_requirements": "torch2vk_b200.runtime.execution_requirements",
    "torch2vk.quantize": "torch2vk_b200.quantize",
}


def install() -> None:
    """Registers the aliases; refuses if a different torch2vk is already imported."""
    existing = sys.modules.get("torch2vk")
    if existing is not None and not getattr(existing, "__torch2vk_b200__", False):
        raise RuntimeError("another torch2vk package is already imported; install() must run first")
    for pkg in ("torch2vk", "torch2vk.runtime", "torch2vk.vulkan"):
        if pkg not in sys.modules:
            mod = types.ModuleType(pkg)
            mod.__path__ = []
            mod.__torch2vk_b200__ = True
            sys.modules[pkg] = mod
    for alias, target in ALIASES.items():
        module = importlib.import_module(target)
        sys.modules[alias] = module
        parent, _, leaf = alias.rpartition(".")
        setattr(sys.modules[parent], leaf, module)
    sys.modules["torch2vk"].runtime = sys.modules["torch2vk.runtime"]
    sys.modules["torch2vk"].vulkan = sys.modules["torch2vk.vulkan"]

"""A RuntimeSession that validates and records dispatches without a GPU (test helper).

It keeps every rule of RuntimeSession.dispatch (frames, field / push-constant
checks, dtype / shape-symbol binding, alias and materialization rules) but
backs tensors with `meta` storage and records (variant, class_name, symbols,
push constants) instead of launching kernels.  It computes nothing.
"""

from __future__ import annotations

import torch

from torch2vk_b200.runtime import optable
from torch2vk_b200.runtime.logical import collect_named_logical_tensors
from torch2vk_b200.runtime.session import TORCH_DTYPES, RuntimeSession
from torch2vk_b200.runtime.types import concrete_shape


class DrySession(RuntimeSession):
    def __init__(self, model_tensors=None) -> None:  # noqa: D107 - no CUDA on purpose
        if model_tensors is not None:
            collect_named_logical_tensors(model_tensors)
        self._model_tensors = model_tensors
        self._get_shader = None
        self._inputs = {}
        self._request_active = False
        self._frame_stack = []
        self._frame_history = {}
        self._dispatch_records = []
        self._checkpoints = {}
        self._weight_cache = {}
        self._request_tensors = set()
        self._frame_tensors = []
        self._closed = False
        self._ops = optable.OPS
        self.device = torch.device("meta")
        self.model_dir = None
        self.profile_dir = None
        self.calls: list[tuple[str, str, dict, dict]] = []

    def _alloc(self, tensor):
        return torch.empty(concrete_shape(tensor.spec), dtype=TORCH_DTYPES[tensor.spec.dtype], device="meta")

    def _materialize_weight(self, tensor):
        with tensor.runtime_write_scope():
            tensor.buffer = self._alloc(tensor)

    def _upload(self, tensor, value):
        with tensor.runtime_write_scope():
            tensor.buffer = self._alloc(tensor)

    def _launch(self, op, variant, buffers, symbols, push_values):
        self.calls.append((variant.name, variant.contract.class_name, dict(symbols), dict(push_values)))

    def synchronize(self) -> None:
        pass

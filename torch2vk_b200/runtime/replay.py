"""Replay plans for RuntimeSession: the reference's replay surface
(src/torch2vk/runtime/replay.py:163-364 ReplayPlan / execute_replay /
stage_replay_step_inputs; session.py:381-408 build_replay_plan /
rebind_replay_plan / replay_plan_compatible / cached_replay_plans /
cache_replay_plan).

The reference pre-records a Vulkan command buffer for a frame and resubmits
it.  Here a plan is the frame's dispatch list as the session recorded it:
for every dispatch the CUDA op, the variant, the LogicalTensor of every field,
the bound shape symbols, the resolved push-constant values and which of them
came from push-constant inputs (those are the plan's dynamic push constants,
e.g. `cache_position`, `start_position`, `token_index`).  The frame released
its workspace at exit, so the plan owns device buffers for every frame-lifetime
tensor it touches; request state, session tensors and weights are bound from
their LogicalTensors.  `execute_replay` re-launches the ops on the session
stream with the dynamic values substituted.  A plan without push-constant
inputs is captured into a CUDA graph on its first execution and replayed from
the graph afterwards (if a capture fails the plan stays on direct launches);
`rebind_replay_plan` drops that graph so the next execution binds the current
buffers.
"""

from __future__ import annotations

import contextlib
from collections.abc import Mapping
from dataclasses import dataclass, field

import numpy as np
import torch

from torch2vk_b200.runtime.logical import LogicalTensor, TensorLifetime, TensorRole
from torch2vk_b200.runtime.shader import PushConstantInput
from torch2vk_b200.runtime.types import concrete_shape, tensor_nbytes


@dataclass
class ReplayDispatch:
    op: object
    variant: object
    tensors: dict[str, LogicalTensor]
    symbols: dict[str, int]
    push_values: dict[str, int | float]
    push_inputs: dict[str, str]  # push-constant field name -> push-constant input name


@dataclass
class ReplayPlan:
    """A frame's dispatches, replayable with new dynamic push-constant values."""

    name: str
    frame: str
    session: object
    dispatches: tuple[ReplayDispatch, ...]
    dynamic_push_constant_names: tuple[str, ...]
    dynamic_symbol_names: tuple[str, ...] = ()
    readback_tensors: dict[str, LogicalTensor] = field(default_factory=dict)
    workspace: dict[int, torch.Tensor] = field(default_factory=dict)  # id(tensor) -> plan-owned buffer
    owned: dict[int, LogicalTensor] = field(default_factory=dict)
    graph: torch.cuda.CUDAGraph | None = None
    graph_failed: bool = False
    _closed: bool = False

    @property
    def num_dispatches(self) -> int:
        return len(self.dispatches)

    @property
    def readback_slots(self) -> dict[str, LogicalTensor]:
        return self.readback_tensors

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        self.graph = None
        self.workspace.clear()
        self.owned.clear()


def _owned(tensor: LogicalTensor) -> bool:
    """Frame workspace and frame inputs are released at frame exit: the plan keeps its own copy."""
    return tensor.lifetime in {TensorLifetime.FRAME, TensorLifetime.OP} and tensor.role is not TensorRole.WEIGHT


def build_replay_plan_impl(rt, *, name: str, frame: str,
                           readback_tensors: Mapping[str, LogicalTensor] | None = None) -> ReplayPlan:
    ctx = rt._frame_history.get(frame)
    if ctx is None:
        raise KeyError(f"no finished frame {frame!r} to build replay plan {name!r} from")
    log = getattr(rt, "_replay_log", [])
    dispatches = tuple(log[ctx.start_dispatch_index:ctx.end_dispatch_index])
    dynamic = sorted({inp for d in dispatches for inp in d.push_inputs.values()})
    plan = ReplayPlan(name=name, frame=frame, session=rt, dispatches=dispatches,
                      dynamic_push_constant_names=tuple(dynamic), readback_tensors=dict(readback_tensors or {}))
    for d in dispatches:
        for t in d.tensors.values():
            root = t
            while root.alias_source is not None:
                root = root.alias_source
            if _owned(root) and id(root) not in plan.workspace:
                plan.workspace[id(root)] = rt._alloc(root)
                plan.owned[id(root)] = root
    return plan


def _buffer(rt, plan: ReplayPlan, tensor: LogicalTensor) -> torch.Tensor:
    if tensor.alias_source is not None:
        src = _buffer(rt, plan, tensor.alias_source)
        nbytes = tensor.alias_nbytes or tensor_nbytes(tensor.spec)
        raw = src.reshape(-1).view(torch.uint8)[tensor.alias_byte_offset:tensor.alias_byte_offset + nbytes]
        from torch2vk_b200.runtime.session import TORCH_DTYPES

        return raw.view(TORCH_DTYPES[tensor.spec.dtype]).reshape(concrete_shape(tensor.spec))
    owned = plan.workspace.get(id(tensor))
    if owned is not None:
        return owned
    if tensor.buffer is None:
        rt._materialize_read(tensor)
    return tensor.buffer


def _on_stream(rt):
    stream = getattr(rt, "stream", None)
    return torch.cuda.stream(stream) if isinstance(stream, torch.cuda.Stream) else contextlib.nullcontext()


def _refresh_inputs(rt, plan: ReplayPlan) -> None:
    """Plan-owned input tensors take the latest registered host values (pinned-free H2D copies)."""
    for key, tensor in plan.owned.items():
        if tensor.role is TensorRole.INPUT and tensor in rt._inputs:
            value = rt._inputs[tensor]
            arr = value.detach().cpu() if isinstance(value, torch.Tensor) else torch.from_numpy(
                np.ascontiguousarray(np.asarray(value)))
            dst = plan.workspace[key]
            if arr.dtype != dst.dtype:
                arr = arr.view(dst.dtype) if arr.element_size() == dst.element_size() and \
                    arr.dtype.is_floating_point != dst.dtype.is_floating_point else arr.to(dst.dtype)
            with _on_stream(rt):
                dst.copy_(arr.reshape(dst.shape), non_blocking=False)


def _launch_all(rt, plan: ReplayPlan, push: Mapping[str, int | float]) -> None:
    for d in plan.dispatches:
        values = dict(d.push_values)
        for field_name, input_name in d.push_inputs.items():
            if input_name in push:
                values[field_name] = push[input_name]
        buffers = {n: _buffer(rt, plan, t) for n, t in d.tensors.items()}
        rt._launch(d.op, d.variant, buffers, d.symbols, values)


def execute_replay(plan: ReplayPlan, dynamic_symbols: Mapping[str, int] | None = None,
                   dynamic_push_constants: Mapping[str, int | float] | None = None) -> dict[str, bytes]:
    """Runs the plan's dispatches with the given dynamic push constants; returns the readback bytes."""
    if plan._closed:
        raise RuntimeError("ReplayPlan is closed")
    symbols = dict(dynamic_symbols or {})
    if unexpected := set(symbols) - set(plan.dynamic_symbol_names):
        raise ValueError(f"ReplayPlan {plan.name!r} got unexpected dynamic symbols: {sorted(unexpected)}")
    push = dict(dynamic_push_constants or {})
    if unexpected := set(push) - set(plan.dynamic_push_constant_names):
        raise ValueError(f"ReplayPlan {plan.name!r} got unexpected dynamic push constants: {sorted(unexpected)}")
    rt = plan.session
    _refresh_inputs(rt, plan)
    static = not plan.dynamic_push_constant_names and isinstance(getattr(rt, "stream", None), torch.cuda.Stream)
    if static and plan.graph is not None:
        with torch.cuda.stream(rt.stream):
            plan.graph.replay()
    elif static and not plan.graph_failed:
        _launch_all(rt, plan, push)  # the first run doubles as the warm-up of every op
        rt.stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(graph, stream=rt.stream):
                _launch_all(rt, plan, push)
            plan.graph = graph
        except Exception:
            plan.graph_failed = True
            torch.cuda.synchronize(rt.device)
    else:
        _launch_all(rt, plan, push)
    results: dict[str, bytes] = {}
    if plan.readback_tensors:
        rt.synchronize()
        for name, tensor in plan.readback_tensors.items():
            results[name] = _buffer(rt, plan, tensor).contiguous().view(torch.uint8).cpu().numpy().tobytes()
    return results


def stage_replay_step_inputs(rt, *, plan: ReplayPlan, inputs: Mapping[LogicalTensor, object],
                             write_through: tuple[LogicalTensor, ...] = ()) -> None:
    """Registers new step inputs; the plan copies them into its own input buffers at execution and
    write_through tensors that live outside the plan are written now."""
    for tensor in inputs:
        tensor.validate_declaration()
        if tensor.role is not TensorRole.INPUT:
            raise ValueError(f"{tensor.name} is not an input tensor")
    rt._inputs.update(inputs)
    for tensor in write_through:
        if tensor in inputs and id(tensor) not in plan.workspace and tensor.buffer is not None:
            value = inputs[tensor]
            src = value.detach().cpu() if isinstance(value, torch.Tensor) else torch.from_numpy(
                np.ascontiguousarray(np.asarray(value)))
            with _on_stream(rt):  # in place: a captured graph keeps this address
                tensor.buffer.copy_(src.to(tensor.buffer.dtype).reshape(tensor.buffer.shape))


def rebind_replay_plan_impl(rt, plan: ReplayPlan) -> None:
    """External buffers may have moved (a new request): the next execution binds them afresh."""
    plan.graph = None


def replay_plan_compatible_impl(rt, plan: ReplayPlan) -> bool:
    if plan._closed or plan.session is not rt:
        return False
    for d in plan.dispatches:
        for t in d.tensors.values():
            if t.buffer is not None and tuple(t.buffer.shape) != tuple(concrete_shape(t.spec)):
                return False
    return True


def push_inputs_of(contract) -> dict[str, str]:
    """Push-constant field name -> push-constant input name for a contract."""
    if contract.push_constants is None:
        return {}
    return {f.name: f.value.name for f in contract.push_constants.fields if isinstance(f.value, PushConstantInput)}

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
their LogicalTensors.  `execute_replay` launches the ops on the session
stream with the dynamic values substituted.  Every plan is captured into a
CUDA graph after its first (direct) execution and replayed from the graph
afterwards.  Dynamic push constants reach a captured graph through device
memory: an op that reads such a value on the GPU asks the `DynamicPush`
wrapper it is handed during capture for a slot of the plan's push buffer, and
the plan rewrites the slots from the step's values (one host-to-device copy)
before each replay; an op may attach guards (e.g. `cache_position < S`, where
its direct form takes another branch), and any host use of the value (int(),
float(), comparisons) bakes the captured value in behind an equality guard.
An execution whose values fail a guard, or that names a different set of
dynamic push constants than the capture did, launches the ops directly; after
an equality-guard or name-set failure the plan captures again for the new
values (at most four times, then it warns once and stays on direct launches).
If a capture fails the plan stays on direct launches; `rebind_replay_plan`
drops the graph so the next execution binds the current buffers.
"""

from __future__ import annotations

import contextlib
import warnings
from collections.abc import Mapping
from dataclasses import dataclass, field

import numpy as np
import torch

from torch2vk_b200.runtime.logical import LogicalTensor, TensorLifetime, TensorRole
from torch2vk_b200.runtime.shader import PushConstantInput
from torch2vk_b200.runtime.types import concrete_shape, tensor_nbytes


_PUSH_BUFFER_BYTES = 1 << 16
_MAX_RECAPTURES = 4
_SLOT_ALIGN = 16


class DynamicPush:
    """A dynamic push-constant value as an op sees it while its plan is captured into a CUDA graph."""

    __slots__ = ("_slots", "name", "value")

    def __init__(self, slots: "PushSlots", name: str, value: int | float):
        self._slots, self.name, self.value = slots, name, value

    def device(self, dtype: torch.dtype, count: int = 1, *, ramp: bool = False,
               clamp_max: int | None = None) -> torch.Tensor:
        """A device tensor of `count` elements holding value (+ i when ramp), capped at clamp_max,
        rewritten from each step's value before every replay."""
        return self._slots.slot(self.name, dtype, count, ramp, clamp_max)

    def guard(self, lo: int | float | None = None, hi: int | float | None = None) -> int | float:
        """The graph serves only steps with lo <= value < hi; returns the captured value."""
        self._slots.guards.add((self.name, "range", lo, hi))
        return self.value

    def _bake(self) -> int | float:
        self._slots.guards.add((self.name, "eq", self.value, None))
        return self.value

    def __int__(self) -> int:
        return int(self._bake())

    def __index__(self) -> int:
        return int(self._bake())

    def __float__(self) -> float:
        return float(self._bake())

    def __bool__(self) -> bool:
        return bool(self._bake())

    def __eq__(self, other) -> bool:
        return self._bake() == (other._bake() if isinstance(other, DynamicPush) else other)

    def __ne__(self, other) -> bool:
        return not self.__eq__(other)

    def __lt__(self, other) -> bool:
        return self._bake() < other

    def __le__(self, other) -> bool:
        return self._bake() <= other

    def __gt__(self, other) -> bool:
        return self._bake() > other

    def __ge__(self, other) -> bool:
        return self._bake() >= other

    def __hash__(self) -> int:
        return hash(self._bake())

    def __add__(self, other):
        return self._bake() + other

    __radd__ = __add__

    def __sub__(self, other):
        return self._bake() - other

    def __rsub__(self, other):
        return other - self._bake()

    def __mul__(self, other):
        return self._bake() * other

    __rmul__ = __mul__

    def __floordiv__(self, other):
        return self._bake() // other

    def __mod__(self, other):
        return self._bake() % other

    def __neg__(self):
        return -self._bake()

    def __repr__(self) -> str:
        return f"DynamicPush({self.name}={self.value!r})"


_NP = {torch.int32: np.int32, torch.int64: np.int64, torch.float32: np.float32}


class PushSlots:
    """Device slots of a captured plan's dynamic push constants and the guards of the capture."""

    def __init__(self, device: torch.device):
        self.buffer = torch.zeros(_PUSH_BUFFER_BYTES, dtype=torch.uint8, device=device)
        self.used = 0
        self.slots: dict[tuple, tuple[int, int]] = {}  # (name, dtype, count, ramp, clamp_max) -> (offset, nbytes)
        self.guards: set[tuple] = set()
        self.names: frozenset[str] = frozenset()
        self._staging: list[torch.Tensor] | None = None
        self._events: list[torch.cuda.Event | None] = [None, None]
        self._turn = 0

    def slot(self, name: str, dtype: torch.dtype, count: int, ramp: bool, clamp_max: int | None) -> torch.Tensor:
        if dtype not in _NP:
            raise TypeError(f"push slot dtype {dtype} is not supported")
        key = (name, dtype, int(count), bool(ramp), clamp_max)
        if key not in self.slots:
            nbytes = int(count) * torch.empty((), dtype=dtype).element_size()
            if self.used + nbytes > _PUSH_BUFFER_BYTES:
                raise RuntimeError("replay push buffer is full")
            self.slots[key] = (self.used, nbytes)
            self.used += (nbytes + _SLOT_ALIGN - 1) // _SLOT_ALIGN * _SLOT_ALIGN
        off, nbytes = self.slots[key]
        return self.buffer[off:off + nbytes].view(dtype)

    def admits(self, push: Mapping[str, int | float]) -> bool:
        return self.rejection(push) is None

    def rejection(self, push: Mapping[str, int | float]) -> str | None:
        """None when the captured graph serves these values, else why not: "names" (another set of
        dynamic push constants), "eq" (a value baked in at capture changed) or "range" (a value outside
        the range the captured ops serve, e.g. a cache position past the cache)."""
        if frozenset(push) != self.names:
            return "names"
        for name, kind, a, b in self.guards:
            v = push[name]
            if kind == "eq" and v != a:
                return "eq"
            if kind == "range" and ((a is not None and v < a) or (b is not None and v >= b)):
                return "range"
        return None

    def host_image(self, push: Mapping[str, int | float]) -> np.ndarray:
        img = np.zeros(max(self.used, _SLOT_ALIGN), np.uint8)
        for (name, dtype, count, ramp, clamp_max), (off, nbytes) in self.slots.items():
            vals = np.full(count, push[name], dtype=np.float64 if dtype == torch.float32 else np.int64)
            if ramp:
                vals = vals + np.arange(count)
            if clamp_max is not None:
                vals = np.minimum(vals, clamp_max)
            img[off:off + nbytes] = np.frombuffer(vals.astype(_NP[dtype]).tobytes(), np.uint8)
        return img

    def upload(self, push: Mapping[str, int | float], stream: torch.cuda.Stream) -> None:
        """Writes the slots for this step on `stream` from one of two pinned staging images (an image
        is rewritten only after its previous copy has finished)."""
        img = self.host_image(push)
        if self._staging is None:
            self._staging = [torch.empty(img.size, dtype=torch.uint8).pin_memory() for _ in range(2)]
        i = self._turn
        self._turn ^= 1
        if self._events[i] is not None:
            self._events[i].synchronize()
        self._staging[i].numpy()[:] = img
        with torch.cuda.stream(stream):
            self.buffer[:img.size].copy_(self._staging[i], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
        self._events[i] = ev


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
    push_slots: PushSlots | None = None
    graph_replays: int = 0
    direct_executions: int = 0
    recaptures: int = 0
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
        self.push_slots = None
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


def _launch_all(rt, plan: ReplayPlan, push: Mapping[str, int | float], slots: PushSlots | None = None) -> None:
    for d in plan.dispatches:
        # outputs the plan does not own get their buffers as the original dispatch gave them (a plan
        # instantiated from an on-disk template runs before anything in this session wrote them)
        for f in d.variant.contract.output_fields:
            t = d.tensors[f.name]
            if t.alias_source is None and not _owned(t) and t.buffer is None:
                rt._materialize_write(t, f.io_kind)
        values = dict(d.push_values)
        for field_name, input_name in d.push_inputs.items():
            if input_name in push:
                values[field_name] = DynamicPush(slots, input_name, push[input_name]) if slots is not None \
                    else push[input_name]
        buffers = {n: _buffer(rt, plan, t) for n, t in d.tensors.items()}
        rt._launch(d.op, d.variant, buffers, d.symbols, values)


def _capture(rt, plan: ReplayPlan, push: Mapping[str, int | float]) -> None:
    """Captures the plan's dispatches into a CUDA graph (nothing runs); dynamic values go through slots."""
    rt.stream.synchronize()
    slots = PushSlots(rt.device) if push else None
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph, stream=rt.stream):
            _launch_all(rt, plan, push, slots)
    except Exception:
        plan.graph_failed = True
        torch.cuda.synchronize(rt.device)
        return
    if slots is not None:
        slots.names = frozenset(push)
    plan.graph, plan.push_slots = graph, slots


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
    on_cuda = isinstance(getattr(rt, "stream", None), torch.cuda.Stream)
    slots = plan.push_slots
    if on_cuda and plan.graph is not None and (slots.admits(push) if slots is not None else not push):
        if slots is not None:
            slots.upload(push, rt.stream)
        with torch.cuda.stream(rt.stream):
            plan.graph.replay()
        plan.graph_replays += 1
    else:
        _launch_all(rt, plan, push)  # the first run doubles as the warm-up of every op
        plan.direct_executions += 1
        why = slots.rejection(push) if slots is not None else ("names" if push else None)
        if on_cuda and plan.graph is not None and not plan.graph_failed and why in ("eq", "names"):
            # the captured graph does not admit these values (an op baked one of them in behind an
            # equality guard, or another set of names): capture again for the new values, a bounded
            # number of times, then stay on direct launches and say so once.  Values outside a range
            # guard (a step the captured ops do not serve) just run directly.
            if plan.recaptures < _MAX_RECAPTURES:
                plan.recaptures += 1
                plan.graph, plan.push_slots = None, None
            else:
                plan.graph_failed = True
                warnings.warn(f"ReplayPlan {plan.name!r}: dynamic push constants {sorted(push)} keep failing the "
                              f"captured graph's guards after {_MAX_RECAPTURES} recaptures; further executions "
                              "launch the dispatches directly", RuntimeWarning, stacklevel=2)
        if on_cuda and plan.graph is None and not plan.graph_failed:
            _capture(rt, plan, push)
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
    plan.push_slots = None


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

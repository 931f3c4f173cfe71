"""Replay plans cached across processes (src/torch2vk/runtime/replay_cache.py:28-148).

A cached plan is also written as a template: per dispatch, the shader variant's name, the
logical tensor bound to each field (by name), the shape symbols and the push constants (with
the names of the dynamic ones).  A later session -- another process -- loads the templates of a
namespace and instantiates every template whose variants resolve through the session's
`get_shader` and whose tensors resolve among its named model tensors with the same shape
symbols; the plan then re-issues those dispatches on that session's buffers without the model
code running again.  Templates live in `<artifact_dir>/../replay_templates_v1/<sha256 of the
namespace>.pkl` (as the reference keys them), only for sessions opened with an artifact_dir.
"""

from __future__ import annotations

import hashlib
import pickle
from dataclasses import dataclass
from pathlib import Path

from torch2vk_b200.runtime.replay import ReplayDispatch, ReplayPlan, _owned, push_inputs_of

TEMPLATE_DIR = "replay_templates_v1"


@dataclass(frozen=True)
class ReplayTemplateEntry:
    shader: str
    tensors: tuple[tuple[str, str], ...]  # (field, logical tensor name)
    symbols: tuple[tuple[str, int], ...]
    push_values: tuple[tuple[str, int | float], ...]


@dataclass(frozen=True)
class ReplayPlanTemplate:
    name: str
    frame: str
    dynamic_push_constant_names: tuple[str, ...]
    entries: tuple[ReplayTemplateEntry, ...]


def template_of(plan: ReplayPlan) -> ReplayPlanTemplate:
    entries = []
    for d in plan.dispatches:
        entries.append(ReplayTemplateEntry(
            shader=d.variant.name,
            tensors=tuple(sorted((field, t.name) for field, t in d.tensors.items())),
            symbols=tuple(sorted(d.symbols.items())),
            push_values=tuple(sorted(d.push_values.items()))))
    return ReplayPlanTemplate(name=plan.name, frame=plan.frame,
                              dynamic_push_constant_names=tuple(plan.dynamic_push_constant_names),
                              entries=tuple(entries))


def template_path(rt, namespace: str) -> Path | None:
    artifact_dir = getattr(rt, "artifact_dir", None)
    if artifact_dir is None:
        return None
    digest = hashlib.sha256(namespace.encode("utf-8")).hexdigest()
    return Path(artifact_dir).parent / TEMPLATE_DIR / f"{digest}.pkl"


def load_templates(rt, namespace: str) -> list[ReplayPlanTemplate]:
    path = template_path(rt, namespace)
    if path is None or not path.is_file():
        return []
    with path.open("rb") as handle:
        loaded = pickle.load(handle)
    if not isinstance(loaded, list) or not all(isinstance(t, ReplayPlanTemplate) for t in loaded):
        raise TypeError(f"replay template cache {path} does not hold a list of ReplayPlanTemplate")
    return loaded


def store_template(rt, namespace: str, plan: ReplayPlan) -> None:
    path = template_path(rt, namespace)
    if path is None:
        return
    templates = load_templates(rt, namespace)
    template = template_of(plan)
    if template in templates:
        return
    templates.append(template)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(".tmp")
    with tmp.open("wb") as handle:
        pickle.dump(templates, handle, protocol=pickle.HIGHEST_PROTOCOL)
    tmp.replace(path)


def instantiate(rt, template: ReplayPlanTemplate) -> ReplayPlan | None:
    """The template as a plan of this session, or None where a variant, a tensor or a shape
    symbol does not match this session's model."""
    get_shader = getattr(rt, "_get_shader", None)
    if get_shader is None:
        return None
    named = rt._named_model_tensors()
    dispatches = []
    for e in template.entries:
        try:
            variant = get_shader(e.shader)
        except (KeyError, ValueError):
            return None
        if variant is None or variant.name != e.shader:
            return None
        tensors = {}
        for field, tname in e.tensors:
            t = named.get(tname)
            if t is None:
                return None
            tensors[field] = t
        contract = variant.contract
        if {f.name for f in contract.fields} != set(tensors):
            return None
        try:
            symbols = rt._bind_shape_symbols(contract.fields, tensors)
        except ValueError:
            return None
        if symbols != dict(e.symbols):
            return None
        op = rt._ops.get(contract.class_name)
        if op is None:
            return None
        dispatches.append(ReplayDispatch(op=op, variant=variant, tensors=tensors, symbols=symbols,
                                         push_values=dict(e.push_values), push_inputs=push_inputs_of(contract)))
    plan = ReplayPlan(name=template.name, frame=template.frame, session=rt, dispatches=tuple(dispatches),
                      dynamic_push_constant_names=template.dynamic_push_constant_names)
    for d in plan.dispatches:
        for t in d.tensors.values():
            root = t
            while root.alias_source is not None:
                root = root.alias_source
            if _owned(root) and id(root) not in plan.workspace:
                plan.workspace[id(root)] = rt._alloc(root)
                plan.owned[id(root)] = root
    return plan

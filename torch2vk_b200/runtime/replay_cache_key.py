"""Replay-plan cache keys and lookups (src/torch2vk/runtime/replay_cache_key.py:14-64): the
helpers the reference's run scripts use to find or build a session's cached plan."""

from __future__ import annotations

import hashlib
from pathlib import Path


def source_tree_digest(source_file: str | Path) -> str:
    """16 hex digits of SHA-256 over a model package's entry file and its dispatch / shaders /
    tensors modules (path and content, in a fixed order): a plan built from other code never matches."""
    entry = Path(source_file)
    root = entry.parent
    files = [entry]
    for sub in ("dispatch", "shaders", "tensors"):
        files.extend(sorted((root / sub).glob("*.py")))
    digest = hashlib.sha256()
    for f in files:
        digest.update(str(f.relative_to(root)).encode("utf-8"))
        digest.update(f.read_bytes())
    return digest.hexdigest()[:16]


def replay_cache_namespace(*, name: str, source_digest: str, model_dir: str | Path,
                           shape_key: str | None = None) -> str:
    base = f"{name}:{source_digest}:{Path(model_dir).expanduser().resolve()}"
    return base if shape_key is None else f"{base}:{shape_key}"


def cached_replay_plan(rt, *, namespace: str):
    plans = rt.cached_replay_plans(namespace)
    return plans[0] if plans else None


def build_cached_replay_plan(rt, *, namespace: str, name: str, frame: str, readback_error: str):
    """Builds a plan for `frame` and caches it under `namespace`; a cached plan must not read back."""
    plan = rt.build_replay_plan(name=name, frame=frame)
    if plan.readback_slots:
        plan.close()
        raise RuntimeError(readback_error)
    rt.cache_replay_plan(namespace, plan)
    return plan

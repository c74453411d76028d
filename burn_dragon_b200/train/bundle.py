"""Multi-stage experiment bundles: ordered training stages with dependencies, resumable
at the last completed stage.

Layout and state files follow the reference (burn_dragon_train/src/train/pipeline/
bundle.rs:14-140, bundle_spec.rs:8-90, state.rs:1-125)::

    <bundle root>/bundle_state.json             name, root, latest completed stage, stages
    <bundle root>/stages/<NN>_<name>/stage_state.json
                                     status pending | running | completed | failed,
                                     start / end unix seconds, last error, artifact
    <bundle root>/stages/<NN>_<name>/resolved_config.json

A stage may depend only on earlier stages; its artifact (here the run directory, final
loss and step count of its training run) is handed to later stages, e.g. to initialise
from a dependency's final checkpoint (``init_from``). ``resume_from_last_completed_stage``
skips stages whose state says completed; ``stop_after_stage`` ends the run after the
named stage.
"""

from __future__ import annotations

import json
import os
import time
from dataclasses import dataclass, field
from typing import Any, Callable

STATES = ("pending", "running", "completed", "failed")


@dataclass
class Stage:
    name: str
    configs: list[str] = field(default_factory=list)
    overrides: dict[str, Any] = field(default_factory=dict)
    depends_on: list[str] = field(default_factory=list)
    init_from: str | None = None


@dataclass
class BundleOptions:
    resume_from_last_completed_stage: bool = True
    stop_after_stage: str | None = None


def validate_bundle(name: str, output_dir: str, stages: list[Stage]) -> None:
    if not name.strip():
        raise ValueError("bundle name must not be empty")
    if not output_dir:
        raise ValueError("bundle output_dir must not be empty")
    if not stages:
        raise ValueError("bundle must contain at least one stage")
    seen: dict[str, int] = {}
    for i, st in enumerate(stages):
        if not st.name.strip():
            raise ValueError(f"stages[{i}].name must not be empty")
        if st.name in seen:
            raise ValueError(f"duplicate stage name `{st.name}`")
        deps = list(st.depends_on) + ([st.init_from] if st.init_from else [])
        known = {s.name for s in stages}
        for d in deps:
            if d == st.name:
                raise ValueError(f"stages[{i}].depends_on cannot reference itself")
            if d not in known:
                raise ValueError(f"stages[{i}].depends_on references unknown stage `{d}`")
            if d not in seen:
                raise ValueError(f"stages[{i}].depends_on must point to earlier stages only")
        seen[st.name] = i


def stage_dir(root: str, index: int, name: str) -> str:
    return os.path.join(root, "stages", f"{index:02d}_{name}")


def _read(path: str):
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f)


def _write(path: str, obj) -> None:
    os.makedirs(os.path.dirname(path), exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        json.dump(obj, f, indent=2, default=str)
    os.replace(tmp, path)


def _stage_state(name: str, status: str, started=None, completed=None, error=None, artifact=None) -> dict:
    return {"stage_name": name, "status": status, "started_at_unix_secs": started,
            "completed_at_unix_secs": completed, "last_error": error, "artifact": artifact or {}}


def _bundle_state(name: str, root: str, states: list[dict]) -> dict:
    done = [s["stage_name"] for s in states if s["status"] == "completed"]
    return {"bundle_name": name, "bundle_root": root, "latest_completed_stage": done[-1] if done else None,
            "stages": states}


def completed_artifacts(root: str, stages: list[Stage]) -> dict[str, dict]:
    out = {}
    for i, st in enumerate(stages):
        s = _read(os.path.join(stage_dir(root, i, st.name), "stage_state.json"))
        if s and s.get("status") == "completed":
            out[st.name] = s.get("artifact", {})
    return out


def execute_bundle(name: str, root: str, stages: list[Stage], options: BundleOptions,
                   run_stage: Callable[[int, Stage, str, dict], dict]) -> dict:
    """Run the stages in order; ``run_stage(index, stage, stage_dir, artifacts)`` returns
    the stage's artifact (a JSON-serialisable dict). Returns the bundle state."""
    root = os.path.abspath(root)
    validate_bundle(name, root, stages)
    artifacts = completed_artifacts(root, stages)
    states: list[dict] = []
    for i, st in enumerate(stages):
        sdir = stage_dir(root, i, st.name)
        sp = os.path.join(sdir, "stage_state.json")
        prior = _read(sp)
        if options.resume_from_last_completed_stage and prior and prior.get("status") == "completed":
            artifacts[st.name] = prior.get("artifact", {})
            states.append(prior)
            if options.stop_after_stage == st.name:
                break
            continue
        for d in st.depends_on + ([st.init_from] if st.init_from else []):
            if d not in artifacts:
                raise RuntimeError(f"stage `{st.name}` depends on `{d}`, which has not completed")
        t0 = int(time.time())
        _write(sp, _stage_state(st.name, "running", t0))
        try:
            art = run_stage(i, st, sdir, artifacts)
        except Exception as e:  # recorded, then re-raised
            states.append(_stage_state(st.name, "failed", t0, int(time.time()), str(e)))
            _write(sp, states[-1])
            _write(os.path.join(root, "bundle_state.json"), _bundle_state(name, root, states))
            raise
        states.append(_stage_state(st.name, "completed", t0, int(time.time()), None, art))
        _write(sp, states[-1])
        artifacts[st.name] = art
        _write(os.path.join(root, "bundle_state.json"), _bundle_state(name, root, states))
        if options.stop_after_stage == st.name:
            break
    return _bundle_state(name, root, states)


def load_bundle_spec(path: str) -> tuple[str, str, list[Stage]]:
    """TOML: [bundle] name, output_dir; [[stages]] name, configs, overrides, depends_on,
    init_from. Relative config paths resolve against the spec file's directory."""
    import tomllib

    with open(path, "rb") as f:
        spec = tomllib.load(f)
    base = os.path.dirname(os.path.abspath(path))
    b = spec.get("bundle", {})
    stages = []
    for s in spec.get("stages", []):
        cfgs = [c if os.path.isabs(c) else os.path.join(base, c) for c in s.get("configs", [])]
        stages.append(Stage(s["name"], cfgs, dict(s.get("overrides", {})), list(s.get("depends_on", [])),
                            s.get("init_from")))
    out = b.get("output_dir", "bundle")
    return b.get("name", ""), out if os.path.isabs(out) else os.path.join(base, out), stages


def train_stage(index: int, stage: Stage, sdir: str, artifacts: dict) -> dict:
    """Default stage runner: one ``train()`` run in the stage directory."""
    from ..config import load_training_config
    from .loop import train

    cfg = load_training_config(stage.configs, stage.overrides)
    if stage.init_from:
        cfg.training.init_checkpoint_path = artifacts[stage.init_from]["run_dir"]
    _write(os.path.join(sdir, "resolved_config.json"), {"configs": stage.configs, "overrides": stage.overrides})
    prev = os.environ.get("BURN_DRAGON_RUN_DIR")
    os.environ["BURN_DRAGON_RUN_DIR"] = os.path.join(sdir, "run")
    try:
        res = train(cfg)
    finally:
        if prev is None:
            os.environ.pop("BURN_DRAGON_RUN_DIR", None)
        else:
            os.environ["BURN_DRAGON_RUN_DIR"] = prev
    return {"run_dir": res["run_dir"], "final_loss": res["final_loss"], "steps": res["steps"]}

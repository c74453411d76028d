"""Experiment manifest: ``<run>/experiment_manifest.json`` with the host, the model spec
and one record per launch (time, command line, SHA-256 of the effective config and of
the training contract, launch mode, the checkpoint resumed from and its files, git
revision). Reference: burn_dragon_language/src/train/manifest.rs:14-200 (schema 2).

The training contract is the config with the launch fields (launch mode, resume
directory and checkpoint) cleared. The reference refuses a launch whose contract differs
from the first one; here the launch is recorded with ``contract_changed = true``
instead, because resuming a run to a larger ``max_iters`` is a supported workflow.
"""

from __future__ import annotations

import copy
import hashlib
import json
import os
import platform
import subprocess
import sys
import time

from .checkpoint import _jsonable

FILE_NAME = "experiment_manifest.json"
SCHEMA_VERSION = 2


def _sha(obj) -> str:
    return hashlib.sha256(json.dumps(_jsonable(obj), sort_keys=True).encode()).hexdigest()


def contract_sha256(cfg) -> str:
    c = copy.deepcopy(cfg)
    c.training.launch_mode = None
    c.training.resume_run_dir = None
    c.training.resume_checkpoint_epoch = None
    return _sha(c)


def _git() -> dict:
    def run(*args):
        try:
            out = subprocess.run(["git", *args], capture_output=True, text=True, timeout=5,
                                 cwd=os.path.dirname(os.path.abspath(__file__)))
            return out.stdout.strip() if out.returncode == 0 else None
        except (OSError, subprocess.SubprocessError):
            return None

    status = run("status", "--porcelain")
    return {"sha": run("rev-parse", "HEAD"), "branch": run("rev-parse", "--abbrev-ref", "HEAD"),
            "dirty": None if status is None else bool(status)}


def _host() -> dict:
    mem = None
    try:
        mem = os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")
    except (ValueError, OSError, AttributeError):
        pass
    label = None
    try:
        import torch

        if torch.cuda.is_available():
            label = torch.cuda.get_device_name(0)
    except Exception:  # noqa: BLE001 (a label is optional)
        label = None
    return {"os": platform.system().lower(), "arch": platform.machine(), "logical_cpus": os.cpu_count(),
            "total_memory_bytes": mem, "hardware_label": label}


def write_experiment_manifest(cfg, run_dir: str, run_name: str, backend: str, resumed_step: int | None) -> dict:
    from .. import __version__ as version

    path = os.path.join(run_dir, FILE_NAME)
    contract = contract_sha256(cfg)
    arts = []
    if resumed_step is not None:
        ck = os.path.join(run_dir, "checkpoint")
        for fn in sorted(os.listdir(ck)):
            if any(fn.endswith(f"-{resumed_step}{e}") for e in (".bin", ".bpk", ".json")):
                arts.append({"file_name": fn, "bytes": os.path.getsize(os.path.join(ck, fn))})
    launch = {"unix_time_ms": int(time.time() * 1000), "command": list(sys.argv), "effective_config_sha256": _sha(cfg),
              "training_contract_sha256": contract, "launch_mode": cfg.training.launch_mode,
              "resume_checkpoint_epoch": resumed_step, "checkpoint_artifacts": arts,
              "config_snapshot": "training_config.json", "git": _git()}
    if os.path.isfile(path):
        man = json.load(open(path))
        if man.get("schema_version") != SCHEMA_VERSION:
            raise ValueError(f"experiment manifest {path} has schema {man.get('schema_version')}, "
                             f"expected {SCHEMA_VERSION}")
        if man["run_name"] != run_name or man["backend"] != backend:
            raise ValueError(f"experiment manifest identity mismatch in {path}: existing run/backend="
                             f"{man['run_name']}/{man['backend']}, requested={run_name}/{backend}")
        first = man["launches"][0]["training_contract_sha256"] if man["launches"] else contract
        launch["contract_changed"] = first != contract
    else:
        man = {"schema_version": SCHEMA_VERSION, "package_version": version, "run_name": run_name, "backend": backend,
               "host": _host(), "model_spec": _jsonable(cfg.model), "training_snapshot": "training_config.json",
               "run_config": "config.json", "launches": []}
        launch["contract_changed"] = False
    man["launches"].append(launch)
    with open(path, "w") as f:
        json.dump(man, f, indent=2)
    return man

"""Multi-stage bundles: validation, state files, resume, init from a dependency (CPU)."""

import json
import os

import pytest

from burn_dragon_b200.cli.bundle import main
from burn_dragon_b200.train.bundle import BundleOptions, Stage, execute_bundle, validate_bundle

CFG = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")


def test_validation_rules():
    with pytest.raises(ValueError):
        validate_bundle("b", "out", [])
    with pytest.raises(ValueError):
        validate_bundle("b", "out", [Stage("a"), Stage("a")])
    with pytest.raises(ValueError):
        validate_bundle("b", "out", [Stage("a", depends_on=["b"]), Stage("b")])
    with pytest.raises(ValueError):
        validate_bundle("b", "out", [Stage("a", depends_on=["zz"])])
    validate_bundle("b", "out", [Stage("a"), Stage("b", depends_on=["a"])])


def test_execute_resume_and_failure(tmp_path):
    calls = []

    def run(i, st, sdir, arts):
        calls.append(st.name)
        if st.name == "boom":
            raise RuntimeError("stage failed")
        return {"value": i, "seen": sorted(arts)}

    stages = [Stage("a"), Stage("b", depends_on=["a"]), Stage("boom")]
    with pytest.raises(RuntimeError):
        execute_bundle("bun", str(tmp_path), stages, BundleOptions(), run)
    st = json.load(open(tmp_path / "bundle_state.json"))
    assert [s["status"] for s in st["stages"]] == ["completed", "completed", "failed"]
    assert st["latest_completed_stage"] == "b" and st["stages"][1]["artifact"]["seen"] == ["a"]
    calls.clear()
    st = execute_bundle("bun", str(tmp_path), stages[:2], BundleOptions(), run)
    assert calls == [] and st["latest_completed_stage"] == "b"
    st = execute_bundle("bun", str(tmp_path), stages[:2], BundleOptions(False, "a"), run)
    assert calls == ["a"] and [s["stage_name"] for s in st["stages"]] == ["a"]


def test_bundle_cli_trains_stages_with_init_from(tmp_path, capsys):
    spec = tmp_path / "bundle.toml"
    spec.write_text(f'''
[bundle]
name = "tiny"
output_dir = "{tmp_path / 'out'}"

[[stages]]
name = "pretrain"
configs = ["{os.path.abspath(CFG)}"]
overrides = {{ training = {{ max_iters = 3, checkpoint_interval_iters = 3, block_size = 32 }} }}

[[stages]]
name = "finetune"
configs = ["{os.path.abspath(CFG)}"]
overrides = {{ training = {{ max_iters = 2, block_size = 32 }} }}
init_from = "pretrain"
''')
    main([str(spec)])
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["stages"] == ["pretrain:completed", "finetune:completed"]
    assert os.path.exists(tmp_path / "out" / "stages" / "00_pretrain" / "run" / "checkpoint" / "model-3.bpk")


def test_adamw_then_eggroll_phases(tmp_path, capsys):
    """The reference's AdamW-warmup -> EGGROLL continuation (burn_dragon_language/src/train/
    phased.rs) as a two-stage bundle."""
    spec = tmp_path / "phases.toml"
    spec.write_text(f'''
[bundle]
name = "adamw_eggroll"
output_dir = "{tmp_path / 'out'}"

[[stages]]
name = "adamw"
configs = ["{os.path.abspath(CFG)}"]
overrides = {{ training = {{ max_iters = 2, checkpoint_interval_iters = 2, block_size = 32 }} }}

[[stages]]
name = "eggroll"
configs = ["{os.path.abspath(CFG)}"]
init_from = "adamw"

[stages.overrides.training]
max_iters = 2
block_size = 32

[stages.overrides.optimizer]
name = "eggroll"
learning_rate = 0.01

[stages.overrides.optimizer.eggroll]
sigma = 0.02
population = {{ population_size = 4, rank = 2 }}
''')
    main([str(spec)])
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["stages"] == ["adamw:completed", "eggroll:completed"]
    info = json.load(open(tmp_path / "out" / "stages" / "01_eggroll" / "run" / "run_info.json"))
    assert info["training_path"] == "eggroll"

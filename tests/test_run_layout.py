"""Run-directory layout, validation sampling, generation defaults and the
language-head key (CPU)."""

import json
import os

import pytest

from burn_dragon_b200.config import RunLayoutConfig, training_config_from_dict
from burn_dragon_b200.train import checkpoint as C

CFG = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")


def test_run_root_rules():
    L = RunLayoutConfig
    assert C.run_root_for(L(), ["x/config/language/baselines/large.toml"], base="r") == \
        os.path.join("r", "language", "baselines", "large")
    assert C.run_root_for(L(mirror_config_path=False), ["x/config/language/a.toml"], base="r") == \
        os.path.join("r", "language")
    assert C.run_root_for(L(), ["cfg/config/local/language/exp/z.toml"], base="r") == \
        os.path.join("r", "language", "local", "exp", "z")
    got = C.run_root_for(L(base_dir="b", category="../cat//x", bundle="bb", stage="s1", variant="v"), [], base="r")
    assert got == os.path.join("b", "language", "cat", "x", "bundles", "bb", "stages", "s1", "variants", "v")
    # the last config path under config/<domain> names the category
    assert C.run_root_for(L(), ["config/language/a.toml", "config/language/sub/b.toml", "other/c.toml"],
                          base="r") == os.path.join("r", "language", "sub", "b")


def test_training_run_uses_layout_and_latest_marker(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    monkeypatch.delenv("BURN_DRAGON_RUN_DIR", raising=False)
    main(["--config", CFG, "--set", "training.max_iters=2", "--set", f'run_layout.base_dir="{tmp_path}"',
          "--set", 'run_layout.category="exp"', "--set", 'run_layout.variant="v1"', "--run-name", "r1"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    root = os.path.join(str(tmp_path), "language", "exp", "variants", "v1", "cpu")
    assert os.path.abspath(res["run_dir"]) == os.path.abspath(os.path.join(root, "r1"))
    assert open(os.path.join(root, "latest")).read() == "r1"


def test_fixed_holdout_validation_repeats_the_same_windows(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    base = ["--config", CFG, "--set", "training.max_iters=4", "--set", "training.validation_interval_iters=2",
            "--set", "optimizer.learning_rate=0.0"]
    vals = {}
    for sampling in ("fixed_holdout", "live_source_selection"):
        main(base + ["--set", f'training.validation.sampling="{sampling}"', "--run-name", sampling, "--no-resume"])
        res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        ev = [json.loads(x) for x in open(os.path.join(res["run_dir"], "events", "metrics.jsonl"))]
        vals[sampling] = [e["valid_loss"] for e in ev if "valid_loss" in e]
    # learning rate 0: the model is fixed, so only the windows can change the loss
    assert len(vals["fixed_holdout"]) == 2 and vals["fixed_holdout"][0] == vals["fixed_holdout"][1]
    assert vals["live_source_selection"][0] != vals["live_source_selection"][1]


def test_external_evaluator_skips_validation(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", CFG, "--set", "training.max_iters=2", "--set", "training.validation_interval_iters=1",
          "--set", 'training.validation.execution="external_evaluator"', "--run-name", "ext"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    ev = [json.loads(x) for x in open(os.path.join(res["run_dir"], "events", "metrics.jsonl"))]
    assert not any("valid_loss" in e for e in ev)


def test_language_head_and_generation_keys(tmp_path, monkeypatch, capsys):
    cfg = training_config_from_dict({"model": {"language_head": {"type": "standard_token_classification"}},
                                     "generation": {"prompt": "hi", "output_format": "token_ids"}})
    assert cfg.generation.prompt == "hi" and not cfg.extras
    with pytest.raises(ValueError, match="nca_factorized_patch"):
        training_config_from_dict({"model": {"language_head": {"type": "nca_factorized_patch", "state_count": 2,
                                                                "patch_size": 2}}})
    from burn_dragon_b200.cli.generate import main as gen
    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", CFG, "--set", "training.max_iters=1", "--set", 'generation.output_format="token_ids"',
          "--set", "generation.max_tokens=3", "--run-name", "g"])
    run_dir = json.loads(capsys.readouterr().out.strip().splitlines()[-1])["run_dir"]
    gen(["--run", run_dir, "--prompt", "ab", "--temperature", "0"])
    ids = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert len(ids) == 3 and all(0 <= i < 256 for i in ids)


def test_generation_context_strategy():
    cfg = training_config_from_dict({"training": {"block_size": 64},
                                     "generation": {"context_strategy": {"type": "sliding", "window": 0}}})
    assert cfg.generation.sliding_window(64) == 64
    cfg.generation.context_strategy = {"type": "sliding", "window": 5}
    assert cfg.generation.sliding_window(64) == 5
    assert training_config_from_dict({}).generation.sliding_window(64) is None
    with pytest.raises(ValueError):
        training_config_from_dict({"generation": {"context_strategy": {"type": "ring"}}})


def test_training_sequence_kernel_override_and_context_strategy():
    cfg = training_config_from_dict({"model": {"sequence_kernel": {"memory_system": "linear_attention"}},
                                     "training": {"sequence_kernel_override": {"memory_system": "gated_deltanet2",
                                                                               "executor": "reference"}}})
    assert cfg.model.sequence_memory_system == "gated_deltanet2" and not cfg.extras
    with pytest.raises(ValueError):
        training_config_from_dict({"training": {"context_strategy": {"type": "ring"}}})


def test_generation_tokenizer_sources(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.generate import main as gen
    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", CFG, "--set", "training.max_iters=1", "--set", "generation.max_tokens=3",
          "--set", 'generation.decode_tokenizer={source="config", type="byte"}', "--run-name", "tk"])
    run_dir = json.loads(capsys.readouterr().out.strip().splitlines()[-1])["run_dir"]
    gen(["--run", run_dir, "--prompt", "ab", "--temperature", "0"])
    text = capsys.readouterr().out.strip().splitlines()[-1]
    assert text.startswith("ab")

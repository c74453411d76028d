"""Launch modes, epochs and streaming document length (CPU)."""

import json
import os

import numpy as np
import pytest

from burn_dragon_b200.cli.train import main
from burn_dragon_b200.config import training_config_from_dict

CFG = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")


def _run(capsys, *args):
    main(["--config", CFG, "--set", "training.block_size=32", *args])
    return json.loads(capsys.readouterr().out.strip().splitlines()[-1])


def test_launch_mode_validation():
    with pytest.raises(ValueError, match="requires training.resume_run_dir"):
        training_config_from_dict({"training": {"launch_mode": "resume_exact_run"}})
    with pytest.raises(ValueError, match="cannot be combined"):
        training_config_from_dict({"training": {"launch_mode": "fresh", "resume_run_dir": "x"}})
    with pytest.raises(ValueError, match="init_checkpoint_path"):
        training_config_from_dict({"training": {"launch_mode": "init_from_checkpoint"}})
    with pytest.raises(ValueError):
        training_config_from_dict({"training": {"launch_mode": "sometimes"}})


def test_fresh_resume_exact_and_resume_latest(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    monkeypatch.delenv("BURN_DRAGON_RUN_NAME", raising=False)
    a = _run(capsys, "--set", 'training.launch_mode="fresh"', "--set", "training.max_iters=2",
             "--set", "training.checkpoint_interval_iters=1")
    b = _run(capsys, "--set", 'training.launch_mode="fresh"', "--set", "training.max_iters=2")
    assert a["run_dir"] != b["run_dir"] and a["steps"] == b["steps"] == 2
    # resume the exact run a, from its step-1 checkpoint, up to 4 steps
    c = _run(capsys, "--set", 'training.launch_mode="resume_exact_run"',
             "--set", f'training.resume_run_dir="{a["run_dir"]}"', "--set", "training.resume_checkpoint_epoch=1",
             "--set", "training.max_iters=4", "--set", "training.checkpoint_interval_iters=1")
    assert c["run_dir"] == a["run_dir"] and c["steps"] == 3
    # the run root's latest marker names the last launched run: a (resumed by c, at step 4)
    d = _run(capsys, "--set", 'training.launch_mode="resume_latest_checkpoint_if_present"',
             "--set", "training.max_iters=5")
    assert os.path.abspath(d["run_dir"]) == os.path.abspath(a["run_dir"]) and d["steps"] == 1


def test_init_from_checkpoint_epoch(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    a = _run(capsys, "--set", "training.max_iters=2", "--set", "training.checkpoint_interval_iters=1",
             "--run-name", "src")
    b = _run(capsys, "--set", 'training.launch_mode="init_from_checkpoint"',
             "--set", f'training.init_checkpoint_path="{a["run_dir"]}"', "--set", "training.init_checkpoint_epoch=1",
             "--set", "training.max_iters=1")
    assert b["run_dir"] != a["run_dir"] and b["steps"] == 1


def test_epochs_set_the_step_count_from_the_dataset(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    path = tmp_path / "corpus.bin"
    np.random.default_rng(0).integers(0, 256, 40_000, dtype=np.uint8).tofile(path)
    res = _run(capsys, "--set", 'dataset.type="file"', "--set", f'dataset.path="{path}"',
               "--set", "dataset.train_split_ratio=0.9", "--set", "training.batch_size=4", "--set", "training.epochs=2",
               "--run-name", "ep")
    assert res["steps"] == 2 * (36_000 // (4 * 32))


def test_min_logical_block_size_lengthens_streams(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.train import loop

    seen = {}
    real = loop.StreamingBytes

    def spy(streams, stream_len, chunk, **kw):
        seen["len"] = stream_len
        return real(streams, stream_len, chunk, **kw)

    monkeypatch.setattr(loop, "StreamingBytes", spy)
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    _run(capsys, "--set", 'training.sequence_batching="streaming"', "--set", "training.tbptt_chunk_size=16",
         "--set", "training.min_logical_block_size=70", "--set", "training.max_iters=2", "--run-name", "ml")
    assert seen["len"] == 96  # 70 rounded up to whole 32-token blocks


def test_sequence_state_probe_reports_warm_and_cold(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    res = _run(capsys, "--set", 'training.sequence_batching="streaming"', "--set", "training.tbptt_chunk_size=16",
               "--set", "training.max_iters=2", "--set", "training.validation_interval_iters=2",
               "--set", "training.sequence_state_probe={enabled=true, paired_batches=2, max_rho_slots=1}",
               "--run-name", "probe")
    rep = json.load(open(os.path.join(res["run_dir"], "sequence_state_probe.json")))
    assert rep["paired_batches"] == 2 and rep["warm_loss"] > 0
    assert abs(rep["carry_nll_gain"] - (rep["paired_cold_loss"] - rep["paired_warm_loss"])) < 1e-9
    assert len(rep["state"]) == 1 and rep["state"][0]["present"]
    ev = [json.loads(x) for x in open(os.path.join(res["run_dir"], "events", "metrics.jsonl"))]
    assert any("stream_carry_nll_gain" in e for e in ev)


def test_experiment_manifest_records_each_launch(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    a = _run(capsys, "--set", "training.max_iters=2", "--set", "training.checkpoint_interval_iters=1",
             "--run-name", "man")
    _run(capsys, "--set", "training.max_iters=3", "--set", "training.checkpoint_interval_iters=1", "--run-name", "man")
    man = json.load(open(os.path.join(a["run_dir"], "experiment_manifest.json")))
    assert man["schema_version"] == 2 and man["run_name"] == "man" and man["backend"] == "cpu"
    first, second = man["launches"]
    assert first["resume_checkpoint_epoch"] is None and second["resume_checkpoint_epoch"] == 2
    assert any(x["file_name"] == "model-2.bpk" and x["bytes"] > 0 for x in second["checkpoint_artifacts"])
    assert second["contract_changed"]  # max_iters grew from 2 to 3
    assert len(first["effective_config_sha256"]) == 64


def test_streaming_rejects_step_features_it_does_not_run(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    with pytest.raises(ValueError, match="module_lr_scales"):
        _run(capsys, "--set", 'training.sequence_batching="streaming"', "--set", "training.tbptt_chunk_size=16",
             "--set", 'training.module_lr_scales=[{target="embedding", scale=0.5}]', "--run-name", "bad")

"""Config loading and the CPU training CLI on the tiny BDH config (d64 n2048 h4 L2, 8 x 128, 20 steps)."""
import json
import os

import pytest

from burn_dragon_b200.cli.train import main, parse_set
from burn_dragon_b200.config import load_training_config

CFG = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs")


def test_extends_and_overlays():
    cfg = load_training_config([os.path.join(CFG, "bdh_gpu_scaffold.toml")])
    assert cfg.model.random_scaffold.enabled and cfg.model.random_scaffold.rank == 16
    assert cfg.parallel.mode == "ddp" and cfg.model.latent_total == 32768
    assert cfg.model.rotary_embedding == "rope"
    cfg = load_training_config([os.path.join(CFG, "tiny_cpu.toml")], parse_set(["training.max_iters=3"]))
    assert cfg.training.max_iters == 3 and cfg.model.n_embd == 64


def test_invalid_parallel_combination_rejected(tmp_path):
    p = tmp_path / "bad.toml"
    p.write_text('extends = "%s"\n[parallel]\nmode = "pipeline"\n[training]\ntbptt_chunk_size = 64\n'
                 % os.path.join(CFG, "tiny_cpu.toml").replace("\\", "/"))
    with pytest.raises(ValueError):
        load_training_config([str(p)])


def test_tiny_cpu_training_run_and_resume(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", os.path.join(CFG, "tiny_cpu.toml"), "--set", "training.checkpoint_interval_iters=10",
          "--run-name", "tiny"])
    out = capsys.readouterr().out
    res = json.loads(out.strip().splitlines()[-1])
    losses = [json.loads(line)["loss"] for line in open(os.path.join(res["run_dir"], "events", "metrics.jsonl"))
              if "loss" in line]
    import math

    # uniform random bytes: the loss stays at the entropy floor ln(256)
    assert len(losses) == 4 and all(abs(v - math.log(256)) < 0.05 for v in losses)
    assert os.path.exists(os.path.join(res["run_dir"], "checkpoint", "model-20.bpk"))
    # resume: nothing left to do at max_iters
    main(["--config", os.path.join(CFG, "tiny_cpu.toml"), "--set", "training.checkpoint_interval_iters=10",
          "--run-name", "tiny"])
    res2 = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res2["steps"] == 0


def test_streaming_tbptt_cpu(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", os.path.join(CFG, "tiny_cpu.toml"), "--set", "training.block_size=64",
          "--set", "training.tbptt_chunk_size=16", "--set", "training.tbptt_persist_across_steps=true",
          "--set", 'training.sequence_batching="streaming"', "--set", "training.max_iters=6",
          "--set", "training.log_frequency=3", "--run-name", "tb"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None


def test_tiny_model_learns_a_periodic_stream():
    """The CPU path actually learns: a period-4 byte stream drops well below ln(256)."""
    import torch

    from burn_dragon_b200.config import DragonConfig
    from burn_dragon_b200.train.trainer import Trainer

    cfg = DragonConfig(n_layer=2, n_embd=64, n_head=4, mlp_internal_dim_multiplier=32, dropout=0.0,
                       rotary_embedding="rope")
    tr = Trainer(cfg, "cpu", lr=3e-3, weight_decay=0.0, seed=1)
    base = torch.tensor([7, 100, 42, 200])
    seq = base.repeat(8 * 33 // 4 + 1)[: 8 * 33].view(8, 33)
    first = last = None
    for i in range(20):
        loss = float(tr.step(seq[:, :-1], seq[:, 1:]))
        first = first if first is not None else loss
        last = loss
    assert last < 0.5 * first


def test_layer_loop_variants_train_checkpoint_resume(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    args = ["--config", os.path.join(CFG, "tiny_cpu_variants.toml"), "--set", "training.checkpoint_interval_iters=2",
            "--run-name", "var"]
    main(args)
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None and res["steps"] == 4
    assert os.path.exists(os.path.join(res["run_dir"], "checkpoint", "extra-4.bpk"))
    main(args[:3] + ["training.max_iters=6", "--run-name", "var"])
    res2 = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res2["steps"] == 2
    # streaming TBPTT carries the runtime state (rho + y-neuron state) across chunks
    main(["--config", os.path.join(CFG, "tiny_cpu_variants.toml"), "--set", "training.block_size=32",
          "--set", "training.tbptt_chunk_size=8", "--set", 'training.sequence_batching="streaming"',
          "--run-name", "var_tb"])
    assert json.loads(capsys.readouterr().out.strip().splitlines()[-1])["final_loss"] is not None


def test_continual_backprop_in_training_loop(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", os.path.join(CFG, "tiny_cpu.toml"), "--set", "training.max_iters=8",
          "--set", "training.continual_backprop.enabled=true", "--set", "training.continual_backprop.warmup_steps=0",
          "--set", "training.continual_backprop.maturity_steps=1", "--set",
          "training.continual_backprop.replace_interval_steps=4", "--set",
          "training.continual_backprop.replacement_rate=0.01", "--set",
          "training.continual_backprop.sample_interval_steps=2", "--run-name", "cbp"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    events = [json.loads(line) for line in open(os.path.join(res["run_dir"], "events", "metrics.jsonl"))]
    assert any("cbp_replaced" in e for e in events)


def test_predictive_coding_training_run(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", os.path.join(CFG, "tiny_cpu.toml"), "--set", "training.max_iters=4",
          "--set", 'training.algorithm="predictive_coding"', "--set", "training.block_size=32",
          "--set", "training.local_predictive_coding.inference.steps=2", "--run-name", "pc"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None and res["steps"] == 4


def test_self_distillation_objective_training_run(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", os.path.join(CFG, "tiny_cpu.toml"), "--set", "training.max_iters=3",
          "--set", "training.block_size=32", "--set", 'training.objective.type="sdft_sdpo"', "--run-name", "sd"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None


def test_run_logs_training_path_and_flop_estimate(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.config import load_training_config
    from burn_dragon_b200.train.metrics import theoretical_forward_flops

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", os.path.join(CFG, "tiny_cpu.toml"), "--set", "training.max_iters=1", "--run-name", "fp"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    info = json.load(open(os.path.join(res["run_dir"], "run_info.json")))
    assert info["training_path"] == "pytorch" and info["mode"] == "single"
    tc = load_training_config(os.path.join(CFG, "tiny_cpu.toml"))
    m, bt = tc.model, tc.training.batch_size * tc.training.block_size
    fl = theoretical_forward_flops(m, tc.training.batch_size, tc.training.block_size)
    assert fl["encoder"] == 2 * bt * m.n_embd * m.latent_total * m.n_layer
    assert info["approx_forward_flops"] == fl


def test_train_shorthand_flags(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--training-config", os.path.join(CFG, "tiny_cpu.toml"), "--backend", "cpu", "--seed", "7",
          "--n-layer", "1", "--latent-total", "512", "--batch-size", "2", "--block-size", "16", "--max-iters", "2",
          "--run-name", "sh"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    tc = json.load(open(os.path.join(res["run_dir"], "training_config.json")))
    assert tc["training"]["seed"] == 7 and tc["model"]["n_layer"] == 1
    assert tc["training"]["batch_size"] == 2 and tc["training"]["block_size"] == 16
    assert tc["model"]["mlp_internal_dim_multiplier"] * tc["model"]["n_embd"] == 512


def test_sharded_v2_checkpoint_run_and_resume(tmp_path, monkeypatch, capsys):
    """``[parallel.checkpoint] format = "sharded_v2"``: the model / optimizer records are
    written as per-rank shard files (one rank here) and a resumed run continues from them."""
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    args = ["--config", os.path.join(CFG, "tiny_cpu.toml"), "--set", "training.checkpoint_interval_iters=2",
            "--set", 'parallel.checkpoint={format="sharded_v2"}', "--run-name", "sh"]
    main(args + ["--set", "training.max_iters=4"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    ck = os.path.join(res["run_dir"], "checkpoint")
    assert os.path.exists(os.path.join(ck, "model-4.shard-0-of-1.bpk"))
    assert not os.path.exists(os.path.join(ck, "model-4.bpk"))
    main(args + ["--set", "training.max_iters=6"])
    res2 = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res2["steps"] == 2
    assert os.path.exists(os.path.join(ck, "model-6.shard-0-of-1.bpk"))

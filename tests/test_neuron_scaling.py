"""Neuron scaling: plateau trigger, widening with moments, frozen / ramped base slice (CPU)."""

import json
import os

import torch

from burn_dragon_b200.cli.train import main
from burn_dragon_b200.config import DragonConfig, NeuronScalingConfig, NeuronScalingStabilizationConfig
from burn_dragon_b200.train.neuron_scaling import NeuronScaler
from burn_dragon_b200.train.trainer import Trainer

CFG = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")


def test_scale_event_widens_and_holds_the_base_slice():
    cfg = DragonConfig(n_layer=2, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="alibi", initialization="simple_normal", vocab_size=32)
    tr = Trainer(cfg, "cpu", lr=1e-2, weight_decay=0.0)
    x = torch.randint(0, 32, (2, 8))
    tr.step(x, x)
    m_before = tr.model.store.view(tr.opt.m, "encoder").clone()
    sc = NeuronScaler(NeuronScalingConfig(enabled=True, min_steps_between_scales=0, capacity_patience_epochs=1,
                                          max_latent_total=10_000,
                                          stabilization=NeuronScalingStabilizationConfig(freeze_base_steps=2,
                                                                                         unfreeze_ramp_steps=2)))
    sc.observe_validation(1.0)
    sc.observe_validation(1.0)
    assert sc.should_scale(5, tr.model.cfg)
    with torch.no_grad():
        out_before = tr.model(x)
    sc.scale(tr, 5)
    nh = cfg.latent_per_head
    assert tr.model.cfg.latent_per_head == 2 * nh
    torch.testing.assert_close(tr.model.store.view(tr.opt.m, "encoder")[:, :, :nh], m_before)
    with torch.no_grad():
        torch.testing.assert_close(tr.model(x), out_before, rtol=1e-5, atol=1e-5)  # function preserved (ALiBi)
    base = tr.model.encoder[:, :, :nh].detach().clone()
    for s in (5, 6):  # frozen
        sc.before_step(tr.model, s)
        tr.step(x, x)
        sc.after_step(s)
        torch.testing.assert_close(tr.model.encoder[:, :, :nh], base)
    sc.before_step(tr.model, 7)  # ramping: half of the optimizer's update lands
    before = tr.model.encoder.detach().clone()
    tr.step(x, x)
    full_update = tr.model.encoder.detach() - before
    sc.after_step(7)
    torch.testing.assert_close(tr.model.encoder[:, :, :nh] - before[:, :, :nh], 0.5 * full_update[:, :, :nh])


def test_training_loop_scales_on_plateau(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", CFG, "--set", "training.max_iters=6", "--set", "training.validation_interval_iters=1",
          "--set", "training.block_size=32", "--set", "training.neuron_scaling.enabled=true",
          "--set", "training.neuron_scaling.min_steps_between_scales=0",
          "--set", "training.neuron_scaling.capacity_patience_epochs=1",
          "--set", "training.neuron_scaling.max_scale_events=1",
          "--set", "training.neuron_scaling.max_latent_total=100000",
          # fresh validation windows each time: their noise makes the plateau the trigger needs
          "--set", 'training.validation.sampling="live_source_selection"', "--run-name", "ns"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    ev = [json.loads(l) for l in open(os.path.join(res["run_dir"], "events", "metrics.jsonl"))]
    scale = [e for e in ev if "neuron_scale_event" in e]
    assert len(scale) == 1 and scale[0]["latent_total"] == 2 * 2048
    assert json.load(open(os.path.join(res["run_dir"], "neuron_scaling.json")))["mlp_internal_dim_multiplier"] == 64

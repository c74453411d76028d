"""Per-module learning-rate scales with schedules (CPU)."""

import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.train.module_lr import ModuleLrScales, ScaleRule
from burn_dragon_b200.train.trainer import Trainer


def test_schedule_rule():
    r = ScaleRule(1.0, {"final_scale": 0.0, "start_fraction": 0.25, "end_fraction": 0.75}, 9)
    assert [r.at(s) for s in (0, 2, 3, 4, 6, 8)] == [1.0, 1.0, 0.75, 0.5, 0.0, 0.0]
    assert ScaleRule(0.3, None, 10).at(5) == 0.3


def test_scales_multiply_the_update():
    cfg = DragonConfig(n_layer=1, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope", vocab_size=32)
    x = torch.randint(0, 32, (2, 8))
    a = Trainer(cfg, "cpu", lr=1e-2, seed=1)
    b = Trainer(cfg, "cpu", lr=1e-2, seed=1)
    e0, h0 = a.model.embed.detach().clone(), a.model.lm_head.detach().clone()
    a.step(x, x)
    mlr = ModuleLrScales([{"target": "embedding", "scale": 0.5}, {"target": "output_head", "scale": 0.0}], 10)
    mlr.before_step(b.model, 0)
    b.step(x, x)
    mlr.after_step(0)
    torch.testing.assert_close(b.model.embed - e0, 0.5 * (a.model.embed - e0))
    torch.testing.assert_close(b.model.lm_head, h0)
    torch.testing.assert_close(b.model.encoder, a.model.encoder)


def test_training_loop_with_module_lr_scales(tmp_path, monkeypatch, capsys):
    import json
    import os

    from burn_dragon_b200.cli.train import main

    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", cfg, "--set", "training.max_iters=3",
          "--set", 'training.module_lr_scales=[{target="embedding", scale=1.0, '
                   'schedule={final_scale=0.0, start_fraction=0.0, end_fraction=1.0}}]',
          "--run-name", "mlr"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None

"""Recurrent-state predictive coding (CPU): cadence, entry-state inference, the
amortisation constraint, the state-only control and a training run."""

import json
import os

import pytest
import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models import reference as R
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.models.state import ModelState
from burn_dragon_b200.train.state_pc import (RecurrentStatePCConfig, amortization_constraint, chunk_due,
                                             correct_entry, state_pc_chunk_loss)


def _setup():
    cfg = DragonConfig(n_layer=2, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, vocab_size=32, dropout=0.0)
    m = BDH(cfg, seed=3)
    g = torch.Generator().manual_seed(0)
    x0 = torch.randint(0, 32, (2, 8), generator=g)
    x = torch.randint(0, 32, (2, 8), generator=g)
    st = ModelState.empty()
    with torch.no_grad():
        m(x0, state=st)
    return m, x, st


def test_cadence():
    c = RecurrentStatePCConfig(enabled=True, apply_every_chunks=3, warmup_steps=1)
    assert [chunk_due(c, i) for i in range(7)] == [False, False, True, False, False, True, False]
    c.observation_contract, c.warmup_steps = "oracle_next_token_negative_control", 0
    assert [chunk_due(c, i) for i in range(4)] == [True, False, False, True]
    with pytest.raises(ValueError, match="allow_oracle_target_leak"):
        c.validate()


def test_entry_inference_lowers_the_observed_energy():
    m, x, st = _setup()
    cfg = RecurrentStatePCConfig(enabled=True, steps=3, step_size=0.5, max_grad_norm=None)

    def energy(rhos):
        with torch.no_grad():
            return float(R.cross_entropy(m(x[:, :-1], state=ModelState(list(rhos), 0)), x[:, 1:]))

    fixed = correct_entry(m, st.rhos, x[:, :-1], x[:, 1:], cfg)
    assert energy(fixed) < energy(st.rhos)


def test_amortization_constraint():
    s = [torch.randn(2, 2, 16, 8)]
    cfg = RecurrentStatePCConfig(amortization_tolerance=0.0, amortization_max_state_slots=4)
    assert float(amortization_constraint(s, [s[0].clone()], cfg, 0)) == 0.0
    c = amortization_constraint(s, [s[0] + 1.0], cfg, 0)
    assert float(c) > 0
    cfg.amortization_tolerance = 10.0  # within tolerance: no pull
    assert float(amortization_constraint(s, [s[0] + 1.0], cfg, 0)) == 0.0


def test_optimizer_mode_adds_the_constraint_and_control_mode_carries_the_teacher():
    m, x, st = _setup()
    cfg = RecurrentStatePCConfig(enabled=True, steps=2, step_size=0.5, amortization_tolerance=0.0)
    y = torch.roll(x, -1, 1)
    base = float(m.loss(x, y, state=ModelState([r.clone() for r in st.rhos], 0)))
    lo, nxt, rep = state_pc_chunk_loss(m, x, y, ModelState([r.clone() for r in st.rhos], 0), cfg, 0)
    assert rep["corrected"] and rep["amortization_loss"] > 0
    assert abs(float(lo) - base - rep["amortization_loss"]) < 1e-5
    cfg.parameter_update = "state_only_control"
    _, nxt2, rep2 = state_pc_chunk_loss(m, x, y, ModelState([r.clone() for r in st.rhos], 0), cfg, 0)
    fixed = correct_entry(m, st.rhos, x[:, :-1], x[:, 1:], cfg)
    replay = ModelState(list(fixed), 0)
    with torch.no_grad():
        m(x, state=replay)
    for a, b in zip(nxt2.rhos, replay.rhos):
        torch.testing.assert_close(a, b)


def test_training_with_recurrent_state_pc(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", cfg, "--set", "training.block_size=32", "--set", 'training.sequence_batching="streaming"',
          "--set", "training.tbptt_chunk_size=16", "--set", "training.max_iters=3",
          "--set", "training.predictive_coding={enabled=true, steps=1, step_size=0.1}", "--run-name", "spc"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None

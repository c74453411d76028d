"""Training-side latent reasoning (CPU): SigReg and JEPA terms against direct
computations, the schedule, rejected options and a training run."""

import json
import os

import pytest
import torch
import torch.nn.functional as F

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.train.latent_reasoning import LatentReasoningTraining

CFG = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu_variants.toml")


def _mc():
    return DragonConfig(n_layer=1, n_embd=8, n_head=2, mlp_internal_dim_multiplier=4, vocab_size=16, dropout=0.0)


def test_schedule_and_rejections():
    lr = LatentReasoningTraining({"enabled": True, "jepa_every_steps": 2, "constraint_balancer":
                                  {"normalized_aux_scale": 2.0, "start_after_steps": 1, "warmup_steps": 4},
                                  "sigreg": {"enabled": False}}, _mc())
    assert lr._scale(0, 2, None) is None  # step 1 is not after start 1
    assert lr._scale(2, 2, None) is None  # step 3 is odd
    assert lr._scale(1, 2, None) is not None and abs(lr._scale(3, 2, None) - 2.0 * 3 / 4) < 1e-9
    with pytest.raises(ValueError):
        LatentReasoningTraining({"next_latent": {"enabled": True}}, _mc())
    with pytest.raises(ValueError):
        LatentReasoningTraining({"start_after_capability_gate_passed": True}, _mc())


def test_sigreg_and_jepa_values():
    torch.manual_seed(0)
    h = torch.randn(2, 6, 8) * 0.3 + 0.2
    lr = LatentReasoningTraining({"jepa_future_offsets": [2], "sigreg": {"min_variance": 0.2,
                                                                         "mean_tolerance": 0.05}}, _mc())
    mean = h.mean((0, 1))
    var = ((h - mean) ** 2).mean((0, 1))
    want = ((0.2 - var).clamp_min(0) ** 2).mean() + ((mean.abs() - 0.05).clamp_min(0) ** 2).mean()
    torch.testing.assert_close(lr.sigreg(h), want)

    class M:
        @staticmethod
        def latent_jepa_prediction(x):
            return 0.5 * x

    got = lr.loss(M(), h, None, 0)
    pred, tgt = 0.5 * h[:, :4], h[:, 2:]
    neg = torch.cat([tgt[1:], tgt[:1]], 0)
    pos = ((pred - tgt) ** 2).mean()
    jepa = pos + F.softplus(pos - ((pred - neg) ** 2).mean() + 1.0)
    torch.testing.assert_close(got, (jepa + want) / 2)


def test_training_run_with_latent_terms(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", CFG, "--set", "training.max_iters=2",
          "--set", 'training.latent_reasoning={enabled=true, target_encoder="ema_teacher", jepa_future_offsets=[1, 2]}',
          "--run-name", "lrt"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None


def test_smooth_l1_fixture_and_next_latent_run(tmp_path, monkeypatch, capsys):
    got = LatentReasoningTraining.smooth_l1(torch.tensor([[[0.5], [3.0]]]), torch.tensor([[[0.0], [1.0]]]), 1.0)
    assert abs(float(got) - 0.8125) < 1e-6  # (0.125 + 1.5) / 2
    with pytest.raises(ValueError, match="next_latent_transition"):
        LatentReasoningTraining({"next_latent": {"enabled": True}}, _mc())
    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", CFG, "--set", "training.max_iters=2", "--set", "model.next_latent_transition={enabled=true}",
          "--set", "training.latent_reasoning={enabled=true, sigreg={enabled=false}, jepa_future_offsets=[], "
                   "next_latent={enabled=true, horizon=2, token_kl_weight=0.5}}",
          "--run-name", "nl"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None


def test_next_latent_term_matches_a_direct_rollout():
    from burn_dragon_b200.models.dragon_runtime import DragonRuntime

    mc = _mc()
    mc.latent_reasoning.enabled = True
    mc.next_latent_transition.enabled = True
    mc.next_latent_transition.zero_init_output = False
    m = DragonRuntime(mc, seed=1)
    tok = torch.randint(0, 16, (2, 5))
    h = m.forward_hidden(tok)
    lr = LatentReasoningTraining({"sigreg": {"enabled": False}, "jepa_future_offsets": [],
                                  "next_latent": {"enabled": True, "horizon": 2}}, mc)
    got = lr.next_latent(m, h, h.detach(), tok)
    emb = m.core.param_dict()["embed"]
    p1 = m.next_latent_prediction(h[:, :4], emb[tok[:, 1:]].detach())
    p2 = m.next_latent_prediction(p1[:, :3], emb[tok[:, 2:]].detach())
    want = (lr.smooth_l1(p1, h[:, 1:].detach(), 1.0) + lr.smooth_l1(p2, h[:, 2:].detach(), 1.0)) / 2
    torch.testing.assert_close(got, want)


def test_energy_model_term_and_run(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.models.dragon_runtime import DragonRuntime

    mc = _mc()
    mc.latent_reasoning.enabled = True
    mc.latent_reasoning.energy_head = True
    mc.latent_reasoning.max_steps = 2
    m = DragonRuntime(mc, seed=2)
    tok = torch.randint(0, 16, (2, 5))
    h = m.forward_hidden(tok)
    lr = LatentReasoningTraining({"sigreg": {"enabled": False}, "jepa_future_offsets": [],
                                  "energy_model": {"enabled": True, "trust_radius": 0.0}}, mc)
    got = lr.energy_model(m, h, h.detach())
    out = m.reason_hidden(h)
    tgt = h.detach()
    neg_e = m.latent_energy(torch.cat([tgt[1:], tgt[:1]], 0))
    prev, terms = m.latent_energy(h), []
    for st, en in zip(out.step_hiddens, out.energies):
        terms += [F.softplus(en - neg_e + 1.0).mean(), 0.25 * (en - prev.detach()).clamp_min(0).mean(),
                  0.05 * ((st - tgt).pow(2).mean().sqrt() / tgt.pow(2).mean().sqrt())]
        prev = en
    torch.testing.assert_close(got, sum(terms) / len(terms))
    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", CFG, "--set", "training.max_iters=2", "--set", "model.latent_reasoning.energy_head=true",
          "--set", "training.latent_reasoning={enabled=true, energy_model={enabled=true}}", "--run-name", "em"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None


def test_step_contract_term_and_run(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.models import reference as R
    from burn_dragon_b200.models.dragon_runtime import DragonRuntime

    mc = _mc()
    mc.latent_reasoning.enabled = True
    mc.latent_reasoning.max_steps = 2
    m = DragonRuntime(mc, seed=4)
    with torch.no_grad():  # a non-zero refiner, so steps move
        m.refiner_out.weight.normal_(0, 0.1)
    tok = torch.randint(0, 16, (2, 5))
    y = torch.randint(0, 16, (2, 5))
    h = m.forward_hidden(tok)
    lr = LatentReasoningTraining({"sigreg": {"enabled": False}, "jepa_future_offsets": [],
                                  "step_contract": {"enabled": True, "ce_weight": 0.5, "trust_radius": 0.0}}, mc)
    got = lr.step_contract(m, h, y)
    out = m.reason_hidden(h)
    prev_h, prev_ce, terms = h.detach(), R.cross_entropy(m.logits_from_hidden(h, 0), y).detach(), []
    for i, st in enumerate(out.step_hiddens):
        ce = R.cross_entropy(m.logits_from_hidden(st, i + 1), y)
        terms += [0.5 * ce, (ce - prev_ce).clamp_min(0),
                  0.05 * (st - prev_h).pow(2).mean().sqrt() / prev_h.pow(2).mean().sqrt()]
        prev_h, prev_ce = st.detach(), ce.detach()
    torch.testing.assert_close(got, sum(terms) / len(terms))
    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", CFG, "--set", "training.max_iters=2",
          "--set", "training.latent_reasoning={enabled=true, step_contract={enabled=true, token_kl_weight=0.1}}",
          "--run-name", "sc"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None

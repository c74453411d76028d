"""Logit entropy floor and repeat unlikelihood (CPU): values against direct
computations, schedule, and a training run that uses them."""

import json
import math
import os

import torch
import torch.nn.functional as F

from burn_dragon_b200.config import LogitEntropyFloorConfig, RepeatUnlikelihoodConfig
from burn_dragon_b200.train.logit_regularizers import (LogitRegularizers, cycle_lags, entropy_floor_loss,
                                                       repeat_unlikelihood_loss, scheduled_weight)


def test_schedule():
    assert scheduled_weight(True, 2.0, 2, 4, 1, 1) == 0.0
    assert scheduled_weight(True, 2.0, 2, 4, 1, 2) == 0.5
    assert scheduled_weight(True, 2.0, 2, 4, 1, 9) == 2.0
    assert scheduled_weight(True, 2.0, 0, 0, 3, 4) == 0.0 and scheduled_weight(True, 2.0, 0, 0, 3, 6) == 2.0
    assert scheduled_weight(False, 2.0, 0, 0, 1, 6) == 0.0


def test_entropy_floor_values():
    torch.manual_seed(0)
    logits = 4 * torch.randn(2, 5, 7)
    y = torch.randint(0, 7, (2, 5))
    lp = F.log_softmax(logits, -1)
    p = lp.exp().reshape(-1, 7)
    cfg = LogitEntropyFloorConfig(enabled=True, weight=1.5, target_entropy_bits=2.5, marginal_weight=0.5,
                                  target_marginal_entropy_bits=2.9, target_coverage_weight=0.25)
    H = -(p * p.log()).sum(1).mean()
    marg = p.mean(0)
    Hm = -(marg * marg.log()).sum()
    want = 1.5 * max(2.5 * math.log(2) - float(H), 0) + 0.5 * max(2.9 * math.log(2) - float(Hm), 0) \
        - 0.25 * float(marg.log()[y.reshape(-1)].mean())
    got = entropy_floor_loss(lp, y, cfg, 0)
    assert abs(float(got) - want) < 1e-5
    # a floor below the current entropy contributes nothing
    cfg2 = LogitEntropyFloorConfig(enabled=True, weight=1.0, target_entropy_bits=0.01)
    assert float(entropy_floor_loss(lp, y, cfg2, 0)) == 0.0


def test_repeat_unlikelihood_values():
    torch.manual_seed(1)
    B, T, V = 2, 6, 5
    logits = torch.randn(B, T, V)
    x = torch.randint(0, V, (B, T))
    y = torch.randint(0, V, (B, T))
    lp = F.log_softmax(logits, -1)
    cfg = RepeatUnlikelihoodConfig(enabled=True, weight=1.0, history_lags=[3], epsilon=1e-4)
    num = hits = 0.0
    for lag in (1, 3):
        for b in range(B):
            for t in range(lag - 1, T):
                h = int(x[b, t - lag + 1])
                if h != int(y[b, t]):
                    pr = min(float(lp[b, t, h].exp()), 1 - 1e-4)
                    num += -math.log(max(1 - pr, 1e-4))
                    hits += 1
    got = repeat_unlikelihood_loss(logits, lp, y, x, cfg, 0)
    assert abs(float(got) - num / max(hits, 1)) < 1e-5
    # cycle margin: softplus(logit[history] - mean logit + margin) on the same mask
    cm = RepeatUnlikelihoodConfig(enabled=True, cycle_margin_weight=2.0, cycle_margin=0.3, cycle_min_lag=2,
                                  cycle_max_lag=2)
    num = hits = 0.0
    for b in range(B):
        for t in range(1, T):
            h = int(x[b, t - 1])
            if h != int(y[b, t]):
                num += float(F.softplus(logits[b, t, h] - logits[b, t].mean() + 0.3))
                hits += 1
    got = repeat_unlikelihood_loss(logits, lp, y, x, cm, 0)
    assert abs(float(got) - 2.0 * num / max(hits, 1)) < 1e-5


def test_cycle_lag_budget_rotates():
    cfg = RepeatUnlikelihoodConfig(cycle_min_lag=2, cycle_max_lag=9, cycle_lags_per_step=3)
    a, b = cycle_lags(cfg, 64, 0), cycle_lags(cfg, 64, 1)
    assert len(a) == 3 and a != b and all(2 <= lag <= 9 for lag in a + b)
    assert cycle_lags(cfg, 4, 0) == [2, 3, 4]


def test_regularized_loss_gradient_raises_entropy():
    torch.manual_seed(2)
    logits = (8 * torch.randn(1, 16, 11)).requires_grad_(True)
    y = torch.randint(0, 11, (1, 16))
    ent = LogitEntropyFloorConfig(enabled=True, weight=1.0, target_entropy_bits=3.0)
    regs = LogitRegularizers(ent, RepeatUnlikelihoodConfig())
    assert regs.active(0)
    with torch.no_grad():
        assert float(regs.loss(logits, y, y, 0)) > float(F.cross_entropy(logits.reshape(-1, 11), y.reshape(-1)))
    floor = entropy_floor_loss(F.log_softmax(logits, -1), y, ent, 0)
    floor.backward()
    H = lambda z: float(-(F.softmax(z, -1) * F.log_softmax(z, -1)).sum(-1).mean())  # noqa: E731
    assert H((logits - 10.0 * logits.grad).detach()) > H(logits.detach()) + 1e-3


def test_training_loop_with_regularizers(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", cfg, "--set", "training.max_iters=4",
          "--set", "training.logit_entropy_floor={enabled=true, weight=0.5, target_entropy_bits=4.0, every_steps=2}",
          "--set", "training.repeat_unlikelihood={enabled=true, weight=0.2, cycle_weight=0.1, warmup_steps=1}",
          "--run-name", "regs"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None and math.isfinite(res["final_loss"])


def test_dynamics_anchor_value_and_masks():
    from burn_dragon_b200.config import DynamicsAnchorConfig
    from burn_dragon_b200.train.logit_regularizers import dynamics_anchor_loss

    torch.manual_seed(3)
    s, t = torch.randn(2, 4, 6), torch.randn(2, 4, 6)
    slp, tlp = F.log_softmax(s, -1), F.log_softmax(t, -1)
    cfg = DynamicsAnchorConfig(enabled=True, weight=2.0, kl="forward")
    kl = (tlp.exp() * (tlp - slp)).sum(-1)
    assert abs(float(dynamics_anchor_loss(slp, t, cfg, 0)) - 2.0 * float(kl.mean())) < 1e-5
    m = torch.tensor([[1, 0, 1, 0], [0, 0, 1, 1]])
    cfg.mask = "context_tokens"
    want = 2.0 * float((kl * (m == 0)).sum() / (m == 0).sum())
    assert abs(float(dynamics_anchor_loss(slp, t, cfg, 0, m)) - want) < 1e-5
    cfg.kl = "jensen_shannon"
    cfg.mask = "all_tokens"
    assert float(dynamics_anchor_loss(slp, s, cfg, 0)) < 1e-6  # identical distributions


def test_training_loop_with_dynamics_anchor(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", cfg, "--set", "training.max_iters=3",
          "--set", "training.dynamics_anchor={enabled=true, weight=0.5, teacher_update_rate=0.1}",
          "--run-name", "anchor"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert math.isfinite(res["final_loss"])


def test_greedy_rollout_prompt_start():
    from burn_dragon_b200.train.logit_regularizers import rollout_prompt_start

    assert rollout_prompt_start(0, 1, 8, 4) == 4  # no span: the window right after one prompt length
    assert [rollout_prompt_start(s, 2, 64, 8) for s in (0, 2, 4, 14)] == [8, 16, 24, 8 + (7 * 8) % 49]
    assert rollout_prompt_start(0, 1, 4, 8) == 0


def test_greedy_rollout_unlikelihood_matches_a_hand_rollout():
    from burn_dragon_b200.config import GreedyRolloutUnlikelihoodConfig
    from burn_dragon_b200.train.logit_regularizers import greedy_rollout_loss

    torch.manual_seed(4)
    V = 5
    W = torch.randn(V, V, requires_grad=True)

    def bigram(tokens, state=None):  # logits of the next token from the current one
        return W[tokens]

    x = torch.tensor([[0, 1, 2, 3, 4, 0, 1, 2], [4, 3, 2, 1, 0, 4, 3, 2]])
    cfg = GreedyRolloutUnlikelihoodConfig(enabled=True, weight=1.0, margin_weight=0.5, margin=0.2, every_steps=1,
                                          prompt_tokens=3, rollout_tokens=4, history_tokens=2, batch_prompts=2,
                                          cycle_min_lag=2, cycle_max_lag=1)
    got = greedy_rollout_loss(bigram, x, cfg, 0)
    # by hand: prompt = x[:, 3:6] (avail 5, min start 3, span 2, step 0)
    u_num = m_num = hits = 0.0
    for b in range(2):
        hist = [int(x[b, 5]), int(x[b, 4])]
        cur = int(x[b, 5])
        for _ in range(4):
            lg = W[cur].detach()
            nxt = int(lg.argmax())
            if nxt in hist:
                p = min(float(torch.softmax(lg, -1)[nxt]), 1 - 1e-4)
                u_num += -math.log(max(1 - p, 1e-4))
                m_num += float(F.softplus(lg[nxt] - lg.mean() + 0.2))
                hits += 1
            hist = [nxt] + hist[:1]
            cur = nxt
    want = (u_num + 0.5 * m_num) / max(hits, 1)
    assert hits > 0 and abs(float(got.detach()) - want) < 1e-5
    got.backward()
    assert W.grad is not None and float(W.grad.abs().sum()) > 0
    assert greedy_rollout_loss(bigram, x, cfg, 1) is not None  # every step
    cfg.every_steps = 4
    assert greedy_rollout_loss(bigram, x, cfg, 2) is None


def test_training_loop_with_greedy_rollout(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", cfg, "--set", "training.max_iters=2",
          "--set", "training.greedy_rollout_unlikelihood={enabled=true, weight=0.5, recovery_weight=0.1, "
                   "sequence_recovery_weight=0.1, entropy_floor_weight=0.1, target_entropy_bits=2.0, every_steps=1, "
                   "prompt_tokens=8, rollout_tokens=3}",
          "--run-name", "rollout"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert math.isfinite(res["final_loss"])


def test_anchor_teacher_is_checkpointed_and_restored(tmp_path, monkeypatch, capsys):
    import torch as T

    from burn_dragon_b200.cli.train import main
    from burn_dragon_b200.train import checkpoint as C

    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    args = ["--config", cfg, "--set", "training.checkpoint_interval_iters=2",
            "--set", "training.dynamics_anchor={enabled=true, weight=0.5, teacher_update_rate=0.5}"]
    main(args + ["--set", "training.max_iters=2", "--run-name", "tch"])
    run_dir = json.loads(capsys.readouterr().out.strip().splitlines()[-1])["run_dir"]
    sd, _ = C.load_tensors(os.path.join(run_dir, "checkpoint", "teacher-model-2.bpk"))
    assert "encoder" in sd and T.isfinite(sd["encoder"]).all()
    main(args + ["--set", "training.max_iters=3", "--run-name", "tch"])  # resumes and restores the teacher
    assert os.path.exists(os.path.join(run_dir, "checkpoint", "teacher-model-3.bpk"))
    from burn_dragon_b200.config import load_training_config
    from burn_dragon_b200.models.bdh import BDH

    fresh = BDH(load_training_config(cfg).model, seed=99)
    assert C.RunDir(run_dir).load_teacher(2, fresh)
    T.testing.assert_close(dict(fresh.named_parameters())["encoder"].detach(), sd["encoder"])

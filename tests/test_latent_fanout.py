"""Latent fan-out schedules: per-layer neuron counts and the sliced forward (CPU)."""

import json
import os

import pytest
import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models import reference as R
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.models.bdh_fused import fused_unsupported


def _cfg(**kw):
    return DragonConfig(n_layer=4, n_embd=16, n_head=2, mlp_internal_dim_multiplier=8, vocab_size=32, dropout=0.0,
                        **kw)


def test_schedules():
    late = _cfg(latent_fanout_schedule={"type": "late_layer", "base_latent_total": 32, "last_layers": 1})
    late.validate()
    assert [late.latent_total_for_layer(i) for i in range(4)] == [32, 32, 32, 128]
    geo = _cfg(latent_fanout_schedule={"type": "geometric", "min_latent_total": 16})
    geo.validate()
    # 16 * 8^(l/3) = 16, 32, 64, 128 (already multiples of lcm(16, 2) = 16)
    assert [geo.latent_total_for_layer(i) for i in range(4)] == [16, 32, 64, 128]
    assert fused_unsupported(geo) == "a latent fan-out schedule"
    with pytest.raises(ValueError):
        _cfg(latent_fanout_schedule={"type": "geometric", "min_latent_total": 24}).validate()  # not a multiple of 16
    with pytest.raises(ValueError):
        _cfg(latent_fanout_schedule={"type": "late_layer", "base_latent_total": 32, "last_layers": 0}).validate()


def test_forward_uses_head_prefixes():
    cfg = _cfg(latent_fanout_schedule={"type": "late_layer", "base_latent_total": 32, "last_layers": 2})
    m = BDH(cfg, device="cpu", seed=3)
    x = torch.randint(0, 32, (2, 12))
    p = m.param_dict()
    with torch.no_grad():
        logits = m(x)
        # by hand: layers 0-1 use 16 of the 64 neurons per head, layers 2-3 all of them
        norm = R.make_norm(cfg.norm_kind, p["norm_gamma"], p["norm_beta"], cfg.norm_eps)
        v = norm(p["embed"][x])
        pos = torch.arange(12)
        H, cap = 2, 64
        for layer in range(4):
            nh = 16 if layer < 2 else 64
            dec = torch.cat([p["decoder"][h * cap:h * cap + nh] for h in range(H)])
            fq = R.rope_freqs(cap, cfg.rope_theta)[:nh] if cfg.rotary_embedding == "rope" else None
            v, _, _ = R.bdh_layer(v, p["encoder"][..., :nh].contiguous(), p["encoder_v"][..., :nh].contiguous(), dec,
                                  p["norm_gamma"], p["norm_beta"], eps=cfg.norm_eps, thr=cfg.thresholds()[0],
                                  thr_y=cfg.thresholds()[1], freqs=fq, positions=pos,
                                  decay=R.decay_vector(cfg.decay_slopes()) if cfg.uses_decay() else None, norm=norm)
        want = v @ p["lm_head"]
    torch.testing.assert_close(logits, want)
    # the narrow layers carry narrow states
    from burn_dragon_b200.models.state import ModelState

    st = ModelState.empty()
    with torch.no_grad():
        m(x, state=st)
    assert [r.shape[2] for r in st.rhos] == [16, 16, 64, 64]


def test_training_with_a_fanout_schedule(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    from burn_dragon_b200.config import load_training_config

    tc = load_training_config(cfg)
    q = tc.model._latent_quantum()
    main(["--config", cfg, "--set", "training.max_iters=3",
          "--set", f'model.latent_fanout_schedule={{type="late_layer", base_latent_total={q}, last_layers=1}}',
          "--run-name", "fan"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None

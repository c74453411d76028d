"""Continual backprop: statistics, selection, feature re-initialisation and moment resets (CPU)."""

import pytest
import torch

from burn_dragon_b200.config import ContinualBackpropConfig, DragonConfig
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.train.continual_backprop import ContinualBackprop
from burn_dragon_b200.train.optim import FusedAdamW


def small():
    return DragonConfig(n_layer=2, n_embd=16, n_head=2, mlp_internal_dim_multiplier=2, dropout=0.0,
                        rotary_embedding="rope", initialization="simple_normal", vocab_size=32)


def test_running_average_of_activation_statistics():
    m = small()
    cbp = ContinualBackprop(ContinualBackpropConfig(enabled=True, utility_decay=0.5), m, 1e-3)
    y = torch.zeros(4, 2, 3, m.latent_per_head)
    y[..., 1] = -2.0
    cbp.record(y)
    cbp._fold_batch()
    assert float(cbp.avg[1]) == -1.0 and float(cbp.avg_abs[1]) == 1.0 and float(cbp.avg_abs[0]) == 0.0


def test_selection_replaces_lowest_utility_and_resets_moments():
    m = small()
    model = BDH(m, seed=0)
    opt = FusedAdamW(model.store, lr=1e-3)
    c = ContinualBackpropConfig(enabled=True, maturity_steps=2, warmup_steps=0, replace_interval_steps=4,
                                replacement_rate=1.0, max_replacements_per_interval=2, cooldown_steps=0,
                                sample_interval_steps=1)
    cbp = ContinualBackprop(c, m, 1e-3)
    Nh = m.latent_per_head
    with torch.no_grad():
        opt.m.fill_(1.0)
        opt.v.fill_(1.0)
    acts = torch.ones(Nh)
    acts[3] = 0.0  # feature 3 never fires
    acts[5] = 0.01
    dec_before = model.decoder.detach().clone()
    enc_before = model.encoder.detach().clone()
    replaced = []
    for _ in range(4):
        cbp.record(acts.view(1, Nh).expand(8, Nh))
        replaced = cbp.after_optimizer_step(model, opt, 1e-3)
    assert sorted(replaced) == [3, 5]
    rows = [h * Nh + f for h in range(m.n_head) for f in (3, 5)]
    assert float(model.decoder[rows].abs().sum()) == 0.0
    keep = [r for r in range(m.latent_total) if r not in rows]
    torch.testing.assert_close(model.decoder[keep], dec_before[keep])
    assert not torch.equal(model.encoder[:, :, 3], enc_before[:, :, 3])
    torch.testing.assert_close(model.encoder[:, :, 0], enc_before[:, :, 0])
    mv = model.store.view(opt.m, "encoder")
    assert float(mv[:, :, 3].abs().sum()) == 0.0 and float(mv[:, :, 0].min()) == 1.0
    assert float(cbp.age[3]) == 0.0 and float(cbp.age[0]) == 4.0
    assert cbp.last.replacement_count == 2


def test_warmup_pause_and_cooldown_block_replacement():
    m = small()
    model = BDH(m, seed=0)
    opt = FusedAdamW(model.store, lr=1e-3)
    c = ContinualBackpropConfig(enabled=True, maturity_steps=0, warmup_steps=4, replace_interval_steps=2,
                                replacement_rate=1.0, cooldown_steps=4)
    cbp = ContinualBackprop(c, m, 1e-3)
    out = [cbp.after_optimizer_step(model, opt, 1e-3) for _ in range(4)]
    assert out == [[], [], [], []] and cbp.last.pause_reason == "warmup"
    cbp.pause(4, "regression")
    cbp.after_optimizer_step(model, opt, 1e-3)
    assert cbp.after_optimizer_step(model, opt, 1e-3) == [] and cbp.last.pause_reason == "regression"
    # lr coupling: half the base lr halves the budget growth
    assert abs(cbp.lr_multiplier(5e-4) - 0.5) < 1e-9


def test_reference_statistics_from_model_forward():
    m = small()
    model = BDH(m, seed=0)
    cbp = ContinualBackprop(ContinualBackpropConfig(enabled=True, utility_decay=0.0), m, 1e-3)
    cbp.record_reference(model, torch.randint(0, 32, (2, 8)))
    cbp._fold_batch()
    assert cbp.samples == m.n_layer and float(cbp.avg_abs.sum()) > 0


@pytest.mark.gpu
def test_statistics_from_fused_step_buffers():
    m = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=16, dropout=0.0,
                     rotary_embedding="rope", initialization="simple_normal", vocab_size=256)
    model = BDH(m, device="cuda", seed=0)
    t = torch.randint(0, 256, (2, 128), device="cuda")
    model.fused_step(t, t)
    cbp = ContinualBackprop(ContinualBackpropConfig(enabled=True, utility_decay=0.0), m, 1e-3)
    cbp.record_fused(model)
    cbp._fold_batch()
    ref = ContinualBackprop(ContinualBackpropConfig(enabled=True, utility_decay=0.0), m, 1e-3)
    ref.record_reference(model, t)
    ref._fold_batch()
    assert cbp.samples == m.n_layer
    torch.testing.assert_close(cbp.avg_abs, ref.avg_abs, rtol=0.05, atol=1e-4)

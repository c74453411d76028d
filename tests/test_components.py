"""Model components beyond the BDH-GPU defaults: norm kinds, PoPE, initialisers."""
import copy
import math

import pytest
import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models import reference as R
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.models.init import init_tensor, near_critical_projection_std


@pytest.mark.parametrize("kind", ["layer_norm", "rms_norm", "dynamic_tanh", "derf"])
def test_norm_kinds_run_and_train(kind):
    cfg = DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope", norm_kind=kind)
    model = BDH(cfg, seed=1)
    x = torch.randint(0, 256, (2, 8))
    loss = model.loss(x, x)
    assert torch.isfinite(loss)
    g = torch.autograd.grad(loss, [model.norm_alpha, model.encoder], allow_unused=True)
    assert g[1] is not None and g[1].abs().sum() > 0
    assert (g[0] is not None) == (kind in ("dynamic_tanh", "derf"))


def test_norm_formulas():
    x = torch.randn(3, 8, dtype=torch.float64)
    g, b = torch.ones(8, dtype=torch.float64), torch.zeros(8, dtype=torch.float64)
    rms = R.make_norm("rms_norm", g, b, 0.0)(x)
    assert torch.allclose(rms.pow(2).mean(-1), torch.ones(3, dtype=torch.float64))
    a = torch.tensor([0.5], dtype=torch.float64)
    assert torch.allclose(R.make_norm("dynamic_tanh", g, b, 0.0, a)(x), torch.tanh(0.5 * x))
    s = torch.tensor([0.1], dtype=torch.float64)
    assert torch.allclose(R.make_norm("derf", g, b, 0.0, a, s)(x), torch.erf(0.5 * x + 0.1))


def test_pope_doubles_latent_and_is_causal_recurrent():
    cfg = DragonConfig(n_layer=1, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="pope")
    model = BDH(cfg, seed=2).double()
    x = torch.randint(0, 256, (1, 6))
    from burn_dragon_b200.models.state import ModelState

    full = model(x)
    st = ModelState.empty()
    parts = [model(x[:, :3], state=st), model(x[:, 3:], state=st)]
    assert torch.allclose(torch.cat(parts, 1), full, atol=1e-9)
    assert st.rhos[0].shape[-2] == 2 * cfg.latent_per_head


@pytest.mark.parametrize("kind", ["simple_normal", "near_critical", "he_glorot", "headwise_semi_orthogonal",
                                  "reservoir"])
def test_initializers(kind):
    g = torch.Generator().manual_seed(0)
    w = init_tensor(kind, "encoder", (2, 64, 256), 64, 256, 6, g)
    assert w.shape == (2, 64, 256) and torch.isfinite(w).all()
    if kind in ("near_critical", "headwise_semi_orthogonal", "reservoir"):
        want = near_critical_projection_std(64, 256) / math.sqrt(6)
        assert abs(float(w.pow(2).mean().sqrt()) - want) < 0.1 * want
    if kind == "headwise_semi_orthogonal":
        m = w[0] / w[0].norm(dim=1, keepdim=True)
        assert torch.allclose(m @ m.t(), torch.eye(64), atol=1e-4)


def test_widen_preserves_function_with_alibi():
    from burn_dragon_b200.models.widen import widen

    cfg = DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="alibi")
    model = BDH(cfg, seed=5).double()
    wide = widen(model.float(), 8).double()
    model = model.double()
    x = torch.randint(0, 256, (2, 9))
    assert wide.cfg.latent_total == 2 * cfg.latent_total
    assert torch.allclose(model(x), wide(x), atol=1e-6)


def test_mhc_sinkhorn_and_training():
    from burn_dragon_b200.models.mhc import sinkhorn

    h = sinkhorn(torch.randn(4, 4), 1.0, 30)
    assert torch.allclose(h.sum(0), torch.ones(4), atol=1e-4) and torch.allclose(h.sum(1), torch.ones(4), atol=1e-4)
    cfg = DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope", mhc_streams=3)
    model = BDH(cfg, seed=1)
    x = torch.randint(0, 256, (2, 8))
    loss = model.loss(x, x)
    g = torch.autograd.grad(loss, [model.mhc_res, model.mhc_post, model.encoder], allow_unused=True)
    assert all(t is not None and torch.isfinite(t).all() for t in g)


def test_mhc_dynamic_positive_controller():
    """dynamic_positive: per-token coefficients from the streams (positive sigmoids, a
    batched Sinkhorn), reference initialisation (zero controller weights, gates at
    sigmoid(-4.59512), carry bias = static h_res logits, bootstrap bias), gradients reach
    the controller, and the TOML key selects it."""
    from burn_dragon_b200.config import training_config_from_dict
    from burn_dragon_b200.models import mhc as MHC

    c = training_config_from_dict({"model": {"n_layer": 2, "n_embd": 32, "n_head": 2,
                                             "mlp_internal_dim_multiplier": 4,
                                             "mhc": {"enabled": True, "num_streams": 3,
                                                     "coefficient_policy": "dynamic_positive"}}}).model
    assert c.mhc_policy == "dynamic_positive" and c.mhc_streams == 3
    cfg = DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope", mhc_streams=3, mhc_policy="dynamic_positive")
    model = BDH(cfg, seed=1)
    assert torch.all(model.mhc_alpha_w == 0) and torch.allclose(model.mhc_carry_gate, torch.tensor(-4.59512))
    assert torch.equal(model.mhc_carry_b.view(2, 3, 3), model.mhc_res)
    assert model.mhc_boot.abs().max() < 1e-3 and model.mhc_boot.abs().max() > 0
    # per-token residual weights are doubly stochastic; branch weights positive
    R = torch.randn(2, 3, 5, 32)
    bi, mixed, w_out = MHC.dynamic_split(R, model.param_dict(), 0, cfg.mhc_tau, 30)
    assert bi.shape == (2, 5, 32) and mixed.shape == R.shape and (w_out > 0).all()
    x = torch.randint(0, 256, (2, 8))
    loss = model.loss(x, x)
    # the controller weights start at zero but are reachable through the gates
    g = torch.autograd.grad(loss, [model.mhc_alpha_w, model.mhc_carry_w, model.mhc_beta_gate, model.encoder])
    assert all(torch.isfinite(t).all() for t in g) and g[0].abs().sum() > 0 and g[1].abs().sum() > 0


def test_initialization_sub_configs_follow_the_reference_rules():
    from burn_dragon_b200.config import training_config_from_dict
    from burn_dragon_b200.models.init import init_param, modular_bridges, projection_std

    # no [model.initialization] table: simple_normal + depth-scaled + heavy-tailed gains
    c = training_config_from_dict({"model": {"n_layer": 4, "n_embd": 32, "n_head": 2,
                                             "mlp_internal_dim_multiplier": 8}}).model
    assert (c.initialization, c.residual_scaling, c.neuron_gains) == ("simple_normal", "depth_scaled",
                                                                       "heavy_tailed_log_normal")
    assert abs(projection_std(c, "encoder", 32, 128) - 0.02 / 2) < 1e-12
    assert projection_std(c, "lm_head", 32, 256) == 0.02
    # a present table takes the sub-tables' own defaults (family_default, iid)
    c2 = training_config_from_dict({"model": {"n_layer": 4, "n_embd": 32, "n_head": 2, "mlp_internal_dim_multiplier": 8,
                                              "initialization": {"kind": "simple_normal"}}}).model
    assert (c2.residual_scaling, c2.neuron_gains) == ("family_default", "iid")
    assert projection_std(c2, "encoder", 32, 128) == 0.02
    g = torch.Generator().manual_seed(0)
    w = init_param(c, "encoder", (2, 32, 128), g)
    col_rms = w.pow(2).mean(1).sqrt()  # per (head, neuron)
    assert float(col_rms.max() / col_rms.min()) > 3.0  # heavy-tailed neuron gains
    # modular bridges: unit RMS, bridge tail on the latent axis
    c3 = copy.deepcopy(c2)
    c3.topology_prior = "modular_bridges"
    m = modular_bridges(c3, 8, 20, "cols")
    assert abs(float(m.pow(2).mean().sqrt()) - 1.0) < 1e-6
    assert torch.allclose(m[:, -1], m[0, -1].expand(8))  # bridge column is constant


def test_firing_target_thresholds():
    from burn_dragon_b200.config import DragonConfig

    c = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=4, firing_targets="gaussian_estimate")
    x, y = c.thresholds()
    assert 0 < x < y  # a rarer y target sits further out in the tail
    c.firing_targets = "explicit_thresholds"
    c.x_firing_threshold, c.y_firing_threshold = 0.1, 0.2
    assert c.thresholds() == (0.1, 0.2)

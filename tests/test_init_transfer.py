"""Initialisation transfer: interface embedding / head, backbone blends and resets (CPU)."""

import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.train.checkpoint import RunDir
from burn_dragon_b200.train.init_transfer import InitTransferConfig, apply_init_transfer


def cfg():
    return DragonConfig(n_layer=2, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                        rotary_embedding="rope", vocab_size=32)


def snap(m):
    return {n: getattr(m, n).detach().clone() for n in m.store.shapes}


def test_backbone_blend_reset_and_preserve(tmp_path):
    loaded = BDH(cfg(), seed=1)
    L = snap(loaded)
    fresh = snap(BDH(cfg(), seed=2))
    apply_init_transfer(loaded, fresh, InitTransferConfig(backbone_blend_alpha=0.25, fresh_top_layers=1,
                                                          preserve_fresh_norm=True))
    torch.testing.assert_close(loaded.decoder, 0.75 * fresh["decoder"] + 0.25 * L["decoder"])
    torch.testing.assert_close(loaded.encoder[1], fresh["encoder"][1])  # last head reset
    torch.testing.assert_close(loaded.encoder[0], 0.75 * fresh["encoder"][0] + 0.25 * L["encoder"][0])
    torch.testing.assert_close(loaded.norm_gamma, fresh["norm_gamma"])
    torch.testing.assert_close(loaded.embed, L["embed"])


def test_match_rms_and_interface_head(tmp_path):
    donor = BDH(cfg(), seed=3)
    RunDir(str(tmp_path / "iface")).save(1, donor)
    m = BDH(cfg(), seed=4)
    with torch.no_grad():
        m.encoder.mul_(7.0)
    head0 = m.lm_head.detach().clone()
    fresh = snap(BDH(cfg(), seed=5))
    apply_init_transfer(m, fresh, InitTransferConfig(interface_checkpoint_path=str(tmp_path / "iface"),
                                                     preserve_interface_input_embedding=True,
                                                     interface_output_head_blend_alpha=0.5, match_fresh_rms=True))
    torch.testing.assert_close(m.embed, donor.embed)
    torch.testing.assert_close(m.lm_head, 0.5 * head0 + 0.5 * donor.lm_head)
    rms = lambda t: float(t.pow(2).mean().sqrt())  # noqa: E731
    assert abs(rms(m.encoder) - rms(fresh["encoder"])) < 1e-5

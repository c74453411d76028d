"""Neuron-dimension widening (burn_dragon_core/src/model/widen.rs; dragon.rs:1268-1534).

Grow the latent size per head Nh -> Nh' keeping each head's existing neurons: the new
encoder columns are zero (so the new x neurons are relu(0 - thr) = 0 and add nothing to
the attention scores nor to the gate), the new encoder_v columns and decoder rows are
fresh draws (their contribution is multiplied by x = 0). With ALiBi (or no rotary
embedding) the widened model computes the same function; RoPE frequencies depend on
Nh, so a RoPE model's existing columns rotate differently after widening.
"""

from __future__ import annotations

import copy

import torch

from .bdh import BDH


@torch.no_grad()
def widen(model: BDH, new_multiplier: int, seed: int = 0) -> BDH:
    cfg = copy.deepcopy(model.cfg)
    if model.cfg.random_scaffold.enabled:
        raise ValueError("widen a dense model (fold the scaffold first)")
    if new_multiplier < cfg.mlp_internal_dim_multiplier:
        raise ValueError("widening cannot shrink the latent size")
    H, Nh, D = cfg.n_head, cfg.latent_per_head, cfg.n_embd
    cfg.mlp_internal_dim_multiplier = new_multiplier
    Nh2 = cfg.latent_per_head
    out = BDH(cfg, device=model.store.data.device, seed=seed)
    out.encoder[:, :, :Nh].copy_(model.encoder)
    out.encoder[:, :, Nh:].zero_()
    out.encoder_v[:, :, :Nh].copy_(model.encoder_v)
    dec_old = model.decoder.view(H, Nh, D)
    out.decoder.view(H, Nh2, D)[:, :Nh].copy_(dec_old)
    for n in ("embed", "lm_head", "norm_gamma", "norm_beta", "norm_alpha", "norm_shift"):
        if n in model.store.shapes:
            getattr(out, n).copy_(getattr(model, n))
    out.store.refresh_shadow()
    return out

"""Initialisation transfer: start a run from another run's weights, adapted.

Reference: ``InitTransferConfig`` (burn_dragon_language/src/config/train/schema.rs:
103-131), applied after loading the init checkpoint (burn_dragon_language/src/
checkpoint.rs:470-560, burn_dragon_core/src/model/dragon/language_head.rs:220-430):

* interface checkpoint (another run directory): take its input embedding and / or LM
  head (``preserve_interface_*``), or blend the head toward it
  (``interface_output_head_blend_alpha``: ``current * (1 - a) + interface * a``);
* backbone adaptation against the fresh initialisation of this run, in order:
  ``match_fresh_rms`` (rescale encoder / encoder_v / decoder / norm to the fresh RMS),
  ``backbone_blend_alpha`` (``fresh * (1 - a) + loaded * a`` for the three projections
  and the norm), ``fresh_top_layers`` (the last k heads of encoder / encoder_v from the
  fresh draw), ``decoder_blend_alpha``, ``norm_blend_alpha``, then
  ``preserve_fresh_decoder`` / ``preserve_fresh_norm``.

``backbone_grad_scale`` is accepted but not applied (the fused step applies AdamW inside
one captured graph with no hook between backward and update).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

BACKBONE = ("encoder", "encoder_v", "decoder")
NORM = ("norm_gamma", "norm_beta", "norm_alpha", "norm_shift")


@dataclass
class InitTransferConfig:
    interface_checkpoint_path: str | None = None
    interface_checkpoint_epoch: int | None = None
    preserve_interface_input_embedding: bool = False
    preserve_interface_output_head: bool = False
    interface_output_head_blend_alpha: float | None = None
    backbone_blend_alpha: float | None = None
    decoder_blend_alpha: float | None = None
    norm_blend_alpha: float | None = None
    backbone_grad_scale: float | None = None
    backbone_grad_scale_steps: int | None = None
    fresh_top_layers: int | None = None
    preserve_fresh_decoder: bool = False
    preserve_fresh_norm: bool = False
    match_fresh_rms: bool = False


def _blend(source: torch.Tensor, fresh: torch.Tensor, alpha: float) -> torch.Tensor:
    a = min(max(alpha, 0.0), 1.0)
    return fresh * (1.0 - a) + source * a


def _rms(t: torch.Tensor) -> float:
    return float(t.double().pow(2).mean().sqrt())


@torch.no_grad()
def apply_init_transfer(model, fresh: dict[str, torch.Tensor], cfg: InitTransferConfig, device=None) -> None:
    """``model``: a ``BDH`` holding the loaded weights; ``fresh``: its parameters as
    initialised before loading (name -> tensor)."""
    names = [n for n in model.store.shapes]
    cur = {n: getattr(model, n) for n in names}
    if cfg.interface_checkpoint_path:
        from ..models.bdh import BDH
        from .checkpoint import RunDir

        donor = BDH(model.cfg, device=model.store.data.device)
        RunDir(cfg.interface_checkpoint_path).load(cfg.interface_checkpoint_epoch, donor, None, device=device)
        if cfg.preserve_interface_input_embedding:
            cur["embed"].copy_(donor.embed)
        if "lm_head" in cur:
            if cfg.preserve_interface_output_head:
                cur["lm_head"].copy_(donor.lm_head)
            if cfg.interface_output_head_blend_alpha:
                cur["lm_head"].copy_(_blend(donor.lm_head, cur["lm_head"], cfg.interface_output_head_blend_alpha))
    present_norm = [n for n in NORM if n in cur]
    if cfg.match_fresh_rms:
        for n in list(BACKBONE) + present_norm:
            s, f = _rms(cur[n]), _rms(fresh[n])
            if s > 1e-8:
                cur[n].mul_(f / s)
    if cfg.backbone_blend_alpha is not None:
        for n in list(BACKBONE) + present_norm:
            cur[n].copy_(_blend(cur[n], fresh[n], cfg.backbone_blend_alpha))
    if cfg.fresh_top_layers:
        k = min(cfg.fresh_top_layers, cur["encoder"].shape[0])
        for n in ("encoder", "encoder_v"):
            cur[n][cur[n].shape[0] - k:].copy_(fresh[n][cur[n].shape[0] - k:])
    if cfg.decoder_blend_alpha is not None:
        cur["decoder"].copy_(_blend(cur["decoder"], fresh["decoder"], cfg.decoder_blend_alpha))
    if cfg.norm_blend_alpha is not None:
        for n in present_norm:
            cur[n].copy_(_blend(cur[n], fresh[n], cfg.norm_blend_alpha))
    if cfg.preserve_fresh_decoder:
        cur["decoder"].copy_(fresh["decoder"])
    if cfg.preserve_fresh_norm:
        for n in present_norm:
            cur[n].copy_(fresh[n])
    model.store.refresh_shadow()

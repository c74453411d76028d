"""Neuron scaling during training: double the latent width when the validation loss
plateaus, then stabilise.

Reference: ``NeuronScalingConfig`` (burn_dragon_language/src/config/train/schema.rs:
151-300) and the widening of every latent-indexed tensor (burn_dragon_core/src/model/
widen.rs; dragon.rs:1268-1534). Rules:

* a scale event fires when the validation loss has not improved for
  ``capacity_patience_epochs`` consecutive validations, at least
  ``min_steps_between_scales`` steps after the previous event, at most
  ``max_scale_events`` times, while the doubled ``latent_total`` stays within
  ``max_latent_total``;
* the model is widened function-preservingly (``models.widen``: new encoder columns
  zero) and the AdamW moments of the existing neurons move with them (new neurons start
  at zero moments);
* stabilisation: for ``freeze_base_steps`` steps the existing neurons' weights are held
  (their update is undone after every optimizer step), then their update is ramped in
  over ``unfreeze_ramp_steps`` up to ``base_lr_scale_after_ramp``; the new neurons'
  updates are scaled by ``new_slice_lr_scale``. Scaling an update after AdamW is the
  per-slice learning-rate multiplier (AdamW's step is invariant to gradient scale).
"""

from __future__ import annotations

import torch

from ..config import NeuronScalingConfig


def _slices(model, nh_old: int):
    """(name, index of the old-neuron slice) of every latent-indexed tensor."""
    H = model.cfg.n_head
    nh = model.cfg.latent_per_head
    dec_rows = (torch.arange(H)[:, None] * nh + torch.arange(nh_old)[None, :]).reshape(-1)
    return [("encoder", (slice(None), slice(None), slice(0, nh_old))),
            ("encoder_v", (slice(None), slice(None), slice(0, nh_old))),
            ("decoder", (dec_rows.to(model.store.data.device),))]


class NeuronScaler:
    def __init__(self, cfg: NeuronScalingConfig):
        self.cfg = cfg
        self.events = 0
        self.last_step = 0
        self.best = float("inf")
        self.stale = 0
        self.scaled_at: int | None = None
        self.nh_old = 0
        self._before: dict[str, torch.Tensor] | None = None
        self._model = None

    # ------------------------------------------------------------ trigger
    def observe_validation(self, loss: float) -> None:
        if loss < self.best - 1e-9:
            self.best, self.stale = loss, 0
        else:
            self.stale += 1

    def should_scale(self, step: int, model_cfg) -> bool:
        c = self.cfg
        return (c.enabled and self.events < c.max_scale_events and self.stale >= c.capacity_patience_epochs
                and step - self.last_step >= c.min_steps_between_scales
                and 2 * model_cfg.latent_total <= c.max_latent_total)

    # ------------------------------------------------------------ the event
    def scale(self, trainer, step: int) -> None:
        """Widen ``trainer.model`` (a ``BDH``) and its optimizer state in place of the old."""
        from ..models.widen import widen
        from .optim import FusedAdamW

        old, opt = trainer.model, trainer.opt
        nh_old = old.cfg.latent_per_head
        new = widen(old, 2 * old.cfg.mlp_internal_dim_multiplier, seed=step)
        nopt = FusedAdamW(new.store, lr=opt.lr, betas=(opt.b1, opt.b2), eps=opt.eps, weight_decay=opt.wd,
                          grad_clip_norm=opt.clip)
        nopt.t = opt.t
        with torch.no_grad():
            for name in new.store.shapes:
                for src, dst in ((opt.m, nopt.m), (opt.v, nopt.v)):
                    a, b = old.store.view(src, name), new.store.view(dst, name)
                    if a.shape == b.shape:
                        b.copy_(a)
                    elif name in ("encoder", "encoder_v"):
                        b[:, :, :nh_old].copy_(a)
                    elif name == "decoder":
                        H, D = old.cfg.n_head, old.cfg.n_embd
                        b.view(H, -1, D)[:, :nh_old].copy_(a.view(H, nh_old, D))
        trainer.model, trainer.opt = new, nopt
        trainer.cfg = new.cfg
        if hasattr(trainer, "_graph"):
            trainer._graph = None
        self.events += 1
        self.last_step = step
        self.stale = 0
        self.scaled_at = step
        self.nh_old = nh_old

    # ------------------------------------------------------------ stabilisation
    def _base_scale(self, step: int) -> float | None:
        if self.scaled_at is None:
            return None
        c = self.cfg.stabilization
        k = step - self.scaled_at
        if k < c.freeze_base_steps:
            return 0.0
        if k < c.freeze_base_steps + c.unfreeze_ramp_steps:
            return c.base_lr_scale_after_ramp * (k - c.freeze_base_steps + 1) / max(c.unfreeze_ramp_steps, 1)
        return c.base_lr_scale_after_ramp

    def active(self, step: int) -> bool:
        s = self._base_scale(step)
        c = self.cfg.stabilization
        return s is not None and (s != 1.0 or c.new_slice_lr_scale != 1.0)

    def before_step(self, model, step: int) -> None:
        self._before = None
        if not self.active(step):
            return
        self._before = {n: getattr(model, n).detach().clone() for n in ("encoder", "encoder_v", "decoder")}
        self._model = model

    def after_step(self, step: int) -> None:
        if self._before is None:
            return
        base = self._base_scale(step)
        new_scale = self.cfg.stabilization.new_slice_lr_scale
        m = self._model
        with torch.no_grad():
            for name, idx in _slices(m, self.nh_old):
                p, b = getattr(m, name), self._before[name]
                upd = p - b
                full = b + upd * new_scale  # the new neurons' update scale, everywhere first
                full[idx] = b[idx] + upd[idx] * base  # then the existing neurons' slice
                p.copy_(full)
        m.store.refresh_shadow()
        self._before = None

"""Continual backprop for the shared low-rank neurons (utility-based feature reset).

A feature is one latent index ``l < Nh`` across every head: its incoming weights are
``encoder[:, :, l]`` and ``encoder_v[:, :, l]``, its outgoing weights the decoder rows
``h*Nh + l``. Every ``sample_interval_steps`` optimizer steps the mean and mean-|.| of
the y-neuron activity per feature (over batch, heads, time and layers) update running
averages (decay ``utility_decay``). Every ``replace_interval_steps`` a replacement
budget grows by ``rate * lr_multiplier * eligible * interval`` (eligible = age >=
``maturity_steps``); up to ``floor(budget)`` (capped per interval) lowest-utility
features, utility = avg|y| * outgoing_L1 / max(incoming_L1, eps), are re-drawn from a
fresh initialisation (incoming weights) with the decoder rows zeroed, their AdamW
moments cleared and their age reset. Warm-up, pause and cool-down windows suppress
replacement; an explicit pause (e.g. after a loss regression) lasts
``regression_pause_steps``.

Reference: burn_dragon_train/src/train/continual_backprop.rs:355-665 (state update,
selection, resets), burn_dragon_core/src/model/dragon/continual_backprop.rs:4-330
(statistics, feature metrics, re-initialisation).

The per-feature statistics are reductions over the y-neuron buffers the fused step
already holds (``FusedWorkspace.yn16``) on sampled steps, or over the activations the
PyTorch path returns; the selection runs on the host on a vector of Nh floats.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..config import ContinualBackpropConfig, DragonConfig


@dataclass
class CBPTelemetry:
    optimizer_step: int
    feature_count: int
    eligible_count: int
    replacement_count: int
    replacement_budget: float
    lr_multiplier: float
    paused: bool
    pause_reason: str | None
    utility_min: float = 0.0
    utility_mean: float = 0.0
    utility_max: float = 0.0
    zero_utility_fraction: float = 0.0


class ContinualBackprop:
    def __init__(self, cfg: ContinualBackpropConfig, model_cfg: DragonConfig, base_lr: float, seed: int = 1337):
        self.cfg = cfg
        self.mcfg = model_cfg
        self.base_lr = base_lr
        self.seed = seed
        n = model_cfg.latent_per_head
        self.step = 0
        self.budget = 0.0
        self.age = torch.zeros(n)
        self.avg = torch.zeros(n)
        self.avg_abs = torch.zeros(n)
        self.samples = 0
        self.pause_until = 0
        self.pause_reason: str | None = None
        self.cooldown_until = 0
        self.replacement_rate_scale = 1.0
        self.max_replacements_override: int | None = None
        self._batch: list[tuple[torch.Tensor, torch.Tensor]] = []
        self.last: CBPTelemetry | None = None

    # ------------------------------------------------------------ statistics
    def should_sample(self) -> bool:
        return (self.step + 1) % max(1, self.cfg.sample_interval_steps) == 0

    def record(self, y: torch.Tensor) -> None:
        """y: activations whose last dim is [..., H*Nh] (fused buffers) or [..., Nh]."""
        n = self.mcfg.latent_per_head
        y = y.detach().float().reshape(-1, n)
        self._batch.append((y.mean(0).cpu(), y.abs().mean(0).cpu()))

    def record_fused(self, model) -> None:
        """Statistics from the y-neuron buffers of the last fused step (all layers)."""
        f = getattr(model, "_fused", None)
        if f is None:
            return
        for yn in f.ws.yn16[:self.mcfg.n_layer]:
            self.record(yn)

    @torch.no_grad()
    def record_reference(self, model, tokens: torch.Tensor) -> None:
        """Statistics from a no-grad PyTorch-path forward (CPU training)."""
        from ..models import reference as R

        cfg = self.mcfg
        p = model.param_dict()
        norm = R.make_norm(cfg.norm_kind, p["norm_gamma"], p["norm_beta"], cfg.norm_eps, p.get("norm_alpha"),
                           p.get("norm_shift"))
        v = norm(p["embed"][tokens])
        T = tokens.shape[1]
        freqs = None
        if cfg.rotary_embedding in ("rope", "pope"):
            f = R.rope_freqs if cfg.rotary_embedding == "rope" else R.pope_freqs
            freqs = f(cfg.latent_per_head, cfg.rope_theta, device=v.device)
        decay = R.decay_vector(cfg.decay_slopes(), device=v.device) if cfg.uses_decay() else None
        pos = torch.arange(T, device=v.device)
        for _ in range(cfg.n_layer):
            v, _, aux = R.bdh_layer(v, p["encoder"], p["encoder_v"], p["decoder"], p["norm_gamma"], p["norm_beta"],
                                    eps=cfg.norm_eps, thr=cfg.thresholds()[0], thr_y=cfg.thresholds()[1], freqs=freqs, positions=pos, decay=decay,
                                    norm=norm, pope=cfg.rotary_embedding == "pope")
            self.record(aux["yn"])

    def _fold_batch(self) -> None:
        if not self._batch:
            return
        mean = torch.stack([m for m, _ in self._batch]).mean(0)
        mabs = torch.stack([a for _, a in self._batch]).mean(0)
        self.samples += len(self._batch)
        self._batch.clear()
        k = self.cfg.utility_decay
        self.avg = self.avg * k + mean * (1 - k)
        self.avg_abs = self.avg_abs * k + mabs * (1 - k)

    # ------------------------------------------------------------ control
    def pause(self, steps: int | None = None, reason: str = "paused") -> None:
        self.pause_until = self.step + (self.cfg.regression_pause_steps if steps is None else steps)
        self.pause_reason = reason

    def lr_multiplier(self, lr: float, target_scale: float = 1.0) -> float:
        ratio = max(lr / self.base_lr, 0.0) if self.base_lr > 0 else 1.0
        m = {"none": 1.0, "global_ratio": ratio, "target_group_ratio": ratio * max(target_scale, 0.0)}[
            self.cfg.lr_coupling]
        return m ** max(self.cfg.lr_coupling_power, 0.0)

    @staticmethod
    def feature_metrics(enc: torch.Tensor, enc_v: torch.Tensor, dec: torch.Tensor):
        H, D, Nh = enc.shape
        enc, enc_v, dec = enc.detach(), enc_v.detach(), dec.detach()
        incoming = (enc.abs().sum((0, 1)) + enc_v.abs().sum((0, 1))).float().cpu()
        outgoing = dec.abs().sum(1).view(H, Nh).sum(0).float().cpu()
        return incoming, outgoing

    def _recovery_active(self) -> bool:
        return self.replacement_rate_scale > 1.0 + 1.1920929e-07 or (
            self.max_replacements_override is not None
            and self.max_replacements_override > self.cfg.max_replacements_per_interval)

    def select(self, enc, enc_v, dec, lr: float) -> list[int]:
        c = self.cfg
        mult = self.lr_multiplier(lr)
        eligible = [i for i in range(len(self.age)) if float(self.age[i]) >= c.maturity_steps]
        rec = self._recovery_active()
        reason = None
        if not rec and self.step <= c.warmup_steps:
            reason = "warmup"
        elif not rec and self.step < self.pause_until:
            reason = self.pause_reason or "paused"
        elif not rec and self.step < self.cooldown_until:
            reason = "cooldown"
        tel = CBPTelemetry(self.step, len(self.age), len(eligible), 0, self.budget, mult, reason is not None, reason)
        self.last = tel
        if reason is not None:
            return []
        if self.step >= self.pause_until:
            self.pause_reason = None
        if not eligible:
            return []
        rate = c.replacement_rate * max(self.replacement_rate_scale, 0.0)
        self.budget += rate * mult * len(eligible) * c.replace_interval_steps
        incoming, outgoing = self.feature_metrics(enc, enc_v, dec)
        util = self.avg_abs.clamp_min(0) * outgoing / incoming.clamp_min(c.utility_epsilon)
        ranked = sorted(eligible, key=lambda i: float(util[i]))
        u = util[eligible]
        tel.utility_min, tel.utility_mean, tel.utility_max = float(u.min()), float(u.mean()), float(u.max())
        tel.zero_utility_fraction = float((u <= c.utility_epsilon).float().mean())
        cap = max(1, self.max_replacements_override or c.max_replacements_per_interval)
        n = min(int(self.budget), cap, len(ranked))
        sel = ranked[:n]
        self.budget -= len(sel)
        tel.replacement_count, tel.replacement_budget = len(sel), self.budget
        return sel

    # ------------------------------------------------------------ the step
    def after_optimizer_step(self, model, optimizer, lr: float) -> list[int]:
        """Call once per optimizer step (after the update). ``model`` is a ``BDH``;
        ``optimizer`` the ``FusedAdamW`` over its store. Returns the replaced features."""
        self.step += 1
        self.age += 1
        self._fold_batch()
        if self.step % max(1, self.cfg.replace_interval_steps):
            return []
        enc, enc_v, dec = model.encoder, model.encoder_v, model.decoder
        sel = self.select(enc, enc_v, dec, lr)
        if not sel:
            return []
        self.reinitialize(model, optimizer, sel)
        idx = torch.tensor(sel)
        self.age[idx] = 0
        self.avg[idx] = 0
        self.avg_abs[idx] = 0
        self.cooldown_until = self.step + self.cfg.cooldown_steps
        return sel

    def reinitialize(self, model, optimizer, sel: list[int]) -> None:
        from ..models.init import init_param

        m = self.mcfg
        H, D, Nh, N = m.n_head, m.n_embd, m.latent_per_head, m.latent_total
        gen = torch.Generator().manual_seed(self.seed * 7919 + self.step)
        idx = torch.tensor(sel, device=model.encoder.device)
        rows = (torch.arange(H, device=idx.device)[:, None] * Nh + idx[None, :]).reshape(-1)
        st = model.store
        with torch.no_grad():
            for name in ("encoder", "encoder_v"):
                fresh = init_param(m, name, (H, D, Nh), gen).to(idx.device)
                p = getattr(model, name)
                p[:, :, idx] = fresh[:, :, idx].to(p.dtype)
                for buf in (optimizer.m, optimizer.v):
                    st.view(buf, name)[:, :, idx] = 0
            model.decoder[rows] = 0
            for buf in (optimizer.m, optimizer.v):
                st.view(buf, "decoder")[rows] = 0
        st.refresh_shadow()

    def state_dict(self) -> dict:
        return {"step": self.step, "budget": self.budget, "age": self.age, "avg": self.avg, "avg_abs": self.avg_abs,
                "samples": self.samples, "pause_until": self.pause_until, "cooldown_until": self.cooldown_until}

    def load_state_dict(self, sd: dict) -> None:
        self.step, self.budget = int(sd["step"]), float(sd["budget"])
        self.age, self.avg, self.avg_abs = sd["age"].clone(), sd["avg"].clone(), sd["avg_abs"].clone()
        self.samples = int(sd["samples"])
        self.pause_until, self.cooldown_until = int(sd["pause_until"]), int(sd["cooldown_until"])

"""Training-side latent reasoning: the JEPA future-latent objective and SigReg on the
final hidden states, with their schedules.

Reference: burn_dragon_language/src/train/steps.rs:10316-10370 (schedule and aux
scale), :10436-10600 (the auxiliary loss), :9621-9700 (target encoder, shifted
negatives, SigReg); config schema.rs:780-1080 (LatentReasoningTrainingConfig).

* JEPA: for each offset k in ``jepa_future_offsets`` (0 < k < T) the model's JEPA
  predictor maps the hidden state at t to a prediction of the target hidden at t + k;
  the term is ``E+ + softplus(E+ - E- + energy_margin)`` with E+ the mean squared error
  to the target and E- to a shifted negative (the batch rolled by one, or time rolled by
  one when the batch has one row). Targets are the detached student hiddens, or an EMA
  teacher's (``target_encoder = "ema_teacher"``).
* SigReg on the hidden: ``mean relu(min_variance - var_d)^2 + mean relu(|mean_d| -
  mean_tolerance)^2`` over feature dims d (statistics over batch and time).
* Each term is scaled by ``constraint_balancer.normalized_aux_scale`` (ramped over its
  ``warmup_steps``), active on steps (1-based) that are multiples of its ``every_steps``
  and after its ``start_after_steps``; the total is divided by the number of active
  terms and added to the next-token CE.

Not built here: the next-latent transition, Dragon-state consistency, energy-model and
step-contract terms, SigReg on rho memory slots, and starts gated on the capability gate
of the event crate (the reference's ``burn_ecs``, absent from its repository); enabling
one of them is an error rather than a silent no-op.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

_EPS = 1.1920929e-07


class LatentReasoningTraining:
    def __init__(self, cfg: dict, model_cfg):
        c = dict(cfg)
        self.every = int(c.get("every_steps", 1))
        self.jepa_every = c.get("jepa_every_steps")
        self.jepa_start = c.get("jepa_start_after_steps")
        self.offsets = [int(k) for k in c.get("jepa_future_offsets", [1, 2, 4, 8])]
        self.target_encoder = c.get("target_encoder", "detached_student")
        self.teacher_rate = float(c.get("teacher_update_rate", 0.01))
        sg = dict(c.get("sigreg", {}))
        self.sg_enabled = bool(sg.get("enabled", True))
        self.sg_every, self.sg_start = sg.get("every_steps"), sg.get("start_after_steps")
        self.sg_target = sg.get("target", "hidden")
        self.min_var = float(sg.get("min_variance", 0.2))
        self.mean_tol = float(sg.get("mean_tolerance", 0.05))
        cb = dict(c.get("constraint_balancer", {}))
        self.scale = float(cb.get("normalized_aux_scale", 1.0))
        self.cb_start = int(cb.get("start_after_steps", 0))
        self.cb_warmup = int(cb.get("warmup_steps", 0))
        self.margin = float(model_cfg.latent_reasoning.energy_margin)
        if self.target_encoder not in ("detached_student", "ema_teacher"):
            raise ValueError(f"training.latent_reasoning.target_encoder {self.target_encoder!r}")
        if c.get("start_after_capability_gate_passed") or any(
                p in ("capability_gate", "fixed_step_and_capability_gate")
                for p in (c.get("jepa_start_policy"), sg.get("start_policy"))):
            raise ValueError("latent-reasoning starts gated on the capability gate need the event crate's gate, "
                             "which is not built here")
        for k in ("next_latent", "dragon_state", "energy_model", "step_contract"):
            if dict(c.get(k, {})).get("enabled"):
                raise ValueError(f"training.latent_reasoning.{k} is not implemented here")
        if self.sg_enabled and self.sg_target != "hidden":
            raise ValueError("training.latent_reasoning.sigreg.target: only \"hidden\" is implemented here")
        self.teacher = None

    def attach_teacher(self, model) -> None:
        if self.target_encoder == "ema_teacher":
            from .objectives import EMATeacher

            self.teacher = EMATeacher(model, min(max(self.teacher_rate, 0.0), 1.0))

    def _scale(self, step: int, every, start) -> float | None:
        every = max(int(self.every if every is None else every), 1)
        start = int(self.cb_start if start is None else start)
        cur = step + 1
        if start > 0 and cur <= start:
            return None
        if every > 1 and cur % every:
            return None
        s = max(self.scale, 0.0)
        if self.cb_warmup > 0:
            s *= min(max(cur - start, 1) / self.cb_warmup, 1.0)
        return s if s > _EPS else None

    def active(self, step: int) -> bool:
        return self._scale(step, self.jepa_every, self.jepa_start) is not None or (
            self.sg_enabled and self._scale(step, self.sg_every, self.sg_start) is not None)

    @staticmethod
    def shifted_negative(t: torch.Tensor) -> torch.Tensor:
        if t.shape[0] > 1:
            return torch.cat([t[1:], t[:1]], 0)
        if t.shape[1] > 1:
            return torch.cat([t[:, 1:], t[:, :1]], 1)
        return t

    def sigreg(self, h: torch.Tensor) -> torch.Tensor:
        mean = h.mean(dim=(0, 1))
        var = (h - mean).pow(2).mean(dim=(0, 1))
        return (self.min_var - var).clamp_min(0.0).pow(2).mean() + (mean.abs() - self.mean_tol).clamp_min(0.0).pow(2).mean()

    def loss(self, model, hidden: torch.Tensor, tokens: torch.Tensor, step: int) -> torch.Tensor | None:
        js = self._scale(step, self.jepa_every, self.jepa_start)
        ss = self._scale(step, self.sg_every, self.sg_start) if self.sg_enabled else None
        total, n = None, 0
        B, T, _ = hidden.shape
        if js is not None:
            if self.teacher is not None:
                with torch.no_grad():
                    target = self.teacher.model.forward_hidden(tokens).detach()
            else:
                target = hidden.detach()
            for k in (k for k in self.offsets if 0 < k < T):
                pred = model.latent_jepa_prediction(hidden[:, :T - k])
                tgt = target[:, k:]
                pos = (pred - tgt).pow(2).mean()
                neg = (pred - self.shifted_negative(tgt)).pow(2).mean()
                term = js * (pos + F.softplus(pos - neg + self.margin))
                total, n = (term if total is None else total + term), n + 1
        if ss is not None:
            term = ss * self.sigreg(hidden)
            total, n = (term if total is None else total + term), n + 1
        return None if total is None else total / max(n, 1)

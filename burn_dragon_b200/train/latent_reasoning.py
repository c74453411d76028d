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
* next latent (steps.rs:9847-9927, helpers train/next_latent.rs:7-32): the model's
  transition predicts the hidden at t + 1 from the hidden at t and the embedding of
  token t + 1 (detached by default), rolled out ``horizon`` steps on its own
  predictions; each step adds ``regression_weight`` x smooth-L1(beta) to the target
  hidden and ``token_kl_weight`` x forward KL between the head's distributions of the
  target and the prediction; the sum is averaged over its terms.
* energy model (steps.rs:9929-10010, :1015-1054): over the first
  ``max_rollout_steps_for_loss`` refinement steps of the model's latent reasoning on the
  hidden, ``contrastive_weight`` x softplus(E_step - E(negative) + margin),
  ``monotonic_weight`` x relu(E_step - E_prev(detached) - tolerance) and
  ``contractive_weight`` x relu(rms(step - target) / rms(target) - trust_radius),
  averaged over its terms (E from the model's energy head).
* step contract (steps.rs, latent_step_contract_auxiliary_loss): over the first
  ``max_rollout_steps_for_loss`` refinement steps, ``ce_weight`` x the step's CE (its
  step-conditioned logits), ``monotonic_ce_weight`` x relu(CE_step - CE_prev(detached) -
  ce_tolerance) (CE_0 from the hidden itself), ``token_kl_weight`` x forward KL to the
  final reasoned logits (detached) and ``contractive_weight`` x relu(rms(step - prev) /
  rms(prev) - trust_radius), averaged over its terms.
* SigReg on the hidden: ``mean relu(min_variance - var_d)^2 + mean relu(|mean_d| -
  mean_tolerance)^2`` over feature dims d (statistics over batch and time).
* Each term is scaled by ``constraint_balancer.normalized_aux_scale`` (ramped over its
  ``warmup_steps``), active on steps (1-based) that are multiples of its ``every_steps``
  and after its ``start_after_steps``; the total is divided by the number of active
  terms and added to the next-token CE.

Not built here: the Dragon-state consistency term, SigReg on rho memory slots, and starts gated on the capability gate
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
        nl = dict(c.get("next_latent", {}))
        self.nl_enabled = bool(nl.get("enabled", False))
        self.nl_every, self.nl_start = nl.get("every_steps"), nl.get("start_after_steps")
        self.nl_horizon = int(nl.get("horizon", 1))
        self.nl_reg = max(float(nl.get("regression_weight", 1.0)), 0.0)
        self.nl_kl = max(float(nl.get("token_kl_weight", 0.0)), 0.0)
        self.nl_beta = float(nl.get("smooth_l1_beta", 1.0))
        self.nl_detach = bool(nl.get("detach_action_embedding", True))
        if self.nl_enabled and not model_cfg.next_latent_transition.enabled:
            raise ValueError("training.latent_reasoning.next_latent needs model.next_latent_transition.enabled")
        em = dict(c.get("energy_model", {}))
        self.em_enabled = bool(em.get("enabled", False))
        self.em_every, self.em_start = em.get("every_steps"), em.get("start_after_steps")
        self.em = {k: float(em.get(k, d)) for k, d in (("contrastive_weight", 1.0), ("monotonic_weight", 0.25),
                                                         ("contractive_weight", 0.05), ("margin", 1.0),
                                                         ("monotonic_tolerance", 0.0), ("trust_radius", 1.0))}
        self.em_steps = int(em.get("max_rollout_steps_for_loss", 4))
        if self.em_enabled and not model_cfg.latent_reasoning.energy_head:
            raise ValueError("training.latent_reasoning.energy_model needs model.latent_reasoning.energy_head")
        sc = dict(c.get("step_contract", {}))
        self.sc_enabled = bool(sc.get("enabled", False))
        self.sc_every, self.sc_start = sc.get("every_steps"), sc.get("start_after_steps")
        self.sc = {k: float(sc.get(k, d)) for k, d in (("ce_weight", 0.0), ("token_kl_weight", 0.0),
                                                         ("monotonic_ce_weight", 1.0), ("contractive_weight", 0.05),
                                                         ("ce_tolerance", 0.0), ("trust_radius", 1.0))}
        self.sc_steps = max(int(sc.get("max_rollout_steps_for_loss", 4)), 1)
        for k in ("dragon_state",):
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
        if self.sc_enabled and self._scale(step, self.sc_every, self.sc_start) is not None:
            return True
        if self.em_enabled and self._scale(step, self.em_every, self.em_start) is not None:
            return True
        if self.nl_enabled and self._scale(step, self.nl_every, self.nl_start) is not None:
            return True
        return self._scale(step, self.jepa_every, self.jepa_start) is not None or (
            self.sg_enabled and self._scale(step, self.sg_every, self.sg_start) is not None)

    @staticmethod
    def shifted_negative(t: torch.Tensor) -> torch.Tensor:
        if t.shape[0] > 1:
            return torch.cat([t[1:], t[:1]], 0)
        if t.shape[1] > 1:
            return torch.cat([t[:, 1:], t[:, :1]], 1)
        return t

    @staticmethod
    def smooth_l1(pred, target, beta: float) -> torch.Tensor:
        beta = max(beta, 1e-8)
        a = (pred - target).abs()
        lin = (a - beta).clamp_min(0.0)
        quad = a - lin
        return (quad.pow(2) * (0.5 / beta) + lin).mean()

    def next_latent(self, model, hidden, target, tokens) -> torch.Tensor | None:
        from .objectives import self_distillation_per_token

        B, T, _ = hidden.shape
        if T < 2 or (self.nl_reg <= _EPS and self.nl_kl <= _EPS):
            return None
        embed = model.core.param_dict()["embed"]
        roll, total, n = hidden, None, 0
        for i in range(min(self.nl_horizon, T - 1)):
            rt = T - (i + 1)
            act = embed[tokens[:, i + 1:]]
            if self.nl_detach:
                act = act.detach()
            pred = model.next_latent_prediction(roll[:, :rt], act)
            if pred is None:
                break
            tgt = target[:, i + 1:].detach()
            if self.nl_reg > _EPS:
                term = self.nl_reg * self.smooth_l1(pred, tgt, self.nl_beta)
                total, n = (term if total is None else total + term), n + 1
            if self.nl_kl > _EPS:
                s_lp = F.log_softmax(model.logits_from_hidden(pred).float(), -1)
                t_lp = F.log_softmax(model.logits_from_hidden(tgt).detach().float(), -1)
                term = self.nl_kl * self_distillation_per_token(s_lp, t_lp, "forward").mean()
                total, n = (term if total is None else total + term), n + 1
            roll = pred
        return None if total is None else total / max(n, 1)

    def energy_model(self, model, hidden, target) -> torch.Tensor | None:
        e = self.em
        prev = model.latent_energy(hidden)
        out = model.reason_hidden(hidden)
        if prev is None or not out.step_hiddens or not out.energies:
            return None
        target = target.detach()
        neg_e = model.latent_energy(self.shifted_negative(target).detach())
        tscale = target.pow(2).mean().sqrt().detach().clamp_min(1e-6)
        total, n = None, 0
        for st, en in list(zip(out.step_hiddens, out.energies))[:self.em_steps]:
            terms = []
            if e["contrastive_weight"] > _EPS and neg_e is not None:
                terms.append(e["contrastive_weight"] * F.softplus(en - neg_e + max(e["margin"], 0.0)).mean())
            if e["monotonic_weight"] > _EPS:
                terms.append(e["monotonic_weight"] * (en - prev.detach() - max(e["monotonic_tolerance"], 0.0))
                             .clamp_min(0.0).mean())
            if e["contractive_weight"] > _EPS:
                # clamped: a zero-initialised refiner starts exactly on the target, where
                # the square root's derivative is undefined
                rms = (st - target).pow(2).mean().clamp_min(1e-12).sqrt()
                terms.append(e["contractive_weight"] * (rms / tscale - max(e["trust_radius"], 0.0)).clamp_min(0.0))
            for t in terms:
                total, n = (t if total is None else total + t), n + 1
            prev = en
        return None if total is None else total / max(n, 1)

    @staticmethod
    def _contract(state, ref, trust):
        scale = ref.pow(2).mean().sqrt().detach().clamp_min(1e-6)
        rms = (state - ref).pow(2).mean().clamp_min(1e-12).sqrt()
        return (rms / scale - max(trust, 0.0)).clamp_min(0.0)

    def step_contract(self, model, hidden, targets, mask=None) -> torch.Tensor | None:
        from ..models import reference as R
        from .objectives import self_distillation_per_token

        c = self.sc
        out = model.reason_hidden(hidden)
        if not out.step_hiddens:
            return None
        prev_h = hidden.detach()
        prev_ce = None if targets is None else R.cross_entropy(model.logits_from_hidden(hidden, 0), targets,
                                                               mask).detach()
        ref = None
        if c["token_kl_weight"] > _EPS:
            ref = F.log_softmax(model.logits_from_hidden(out.final_hidden, out.steps_used).detach().float(), -1)
        total, n = None, 0

        def add(t):
            nonlocal total, n
            total, n = (t if total is None else total + t), n + 1

        for i, st in enumerate(out.step_hiddens[:self.sc_steps]):
            lg = model.logits_from_hidden(st, i + 1)
            ce = None if targets is None else R.cross_entropy(lg, targets, mask)
            if c["ce_weight"] > _EPS and ce is not None:
                add(c["ce_weight"] * ce)
            if c["monotonic_ce_weight"] > _EPS and ce is not None and prev_ce is not None:
                add(c["monotonic_ce_weight"] * (ce - (prev_ce + max(c["ce_tolerance"], 0.0))).clamp_min(0.0))
            if ref is not None:
                add(c["token_kl_weight"] * self_distillation_per_token(F.log_softmax(lg.float(), -1), ref,
                                                                        "forward").mean())
            if c["contractive_weight"] > _EPS:
                add(c["contractive_weight"] * self._contract(st, prev_h, c["trust_radius"]))
            prev_h = st.detach()
            if ce is not None:
                prev_ce = ce.detach()
        return None if total is None else total / max(n, 1)

    def sigreg(self, h: torch.Tensor) -> torch.Tensor:
        mean = h.mean(dim=(0, 1))
        var = (h - mean).pow(2).mean(dim=(0, 1))
        return (self.min_var - var).clamp_min(0.0).pow(2).mean() + (mean.abs() - self.mean_tol).clamp_min(0.0).pow(2).mean()

    def loss(self, model, hidden: torch.Tensor, tokens: torch.Tensor, step: int, targets=None,
             mask=None) -> torch.Tensor | None:
        js = self._scale(step, self.jepa_every, self.jepa_start)
        ss = self._scale(step, self.sg_every, self.sg_start) if self.sg_enabled else None
        ns = self._scale(step, self.nl_every, self.nl_start) if self.nl_enabled else None
        es = self._scale(step, self.em_every, self.em_start) if self.em_enabled else None
        total, n = None, 0
        B, T, _ = hidden.shape
        target = None
        if js is not None or ns is not None or es is not None:
            if self.teacher is not None:
                with torch.no_grad():
                    target = self.teacher.model.forward_hidden(tokens).detach()
            else:
                target = hidden.detach()
        if ns is not None:
            term = self.next_latent(model, hidden, target, tokens)
            if term is not None:
                total, n = ns * term, 1
        sc = self._scale(step, self.sc_every, self.sc_start) if self.sc_enabled else None
        if sc is not None:
            term = self.step_contract(model, hidden, targets, mask)
            if term is not None:
                total, n = (sc * term if total is None else total + sc * term), n + 1
        if es is not None:
            term = self.energy_model(model, hidden, target)
            if term is not None:
                total, n = (es * term if total is None else total + es * term), n + 1
        if js is not None:
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

"""Auxiliary next-token losses on the output distribution.

Reference: burn_dragon_language/src/train/steps.rs ``next_token_loss_from_logits``
(:4076-4250) with its helpers (:13048-13090, :13373-13480) and the weight schedule
``scheduled_weight_on_cadence`` (:3390-3422); configs in
burn_dragon_language/src/config/train/schema.rs:340-410.

* logit entropy floor: ``w * relu(H_target - mean_t H(p_t))`` (nats; targets are given
  in bits), the same floor on the batch-marginal distribution ``mean_t p_t`` (log
  clamped at 1e-12), and target coverage ``-mean_t log max(marginal[y_t], eps)``;
* repeat unlikelihood: for each lag ``l`` (1 plus ``history_lags``) the prediction at
  position ``t >= l - 1`` is pushed away from the input token at ``t - l + 1`` with
  ``-log(max(1 - min(p, 1 - eps), eps))``, counted only where that token is not the
  real target; the cycle variant does the same over a rotating budget of lags in
  ``[cycle_min_lag, cycle_max_lag]``, and the cycle margin adds
  ``softplus(logit[history] - mean logit + margin)`` on those positions.

* dynamics anchor: ``w * masked_mean_t D(student_t, teacher_t)`` with D the forward /
  reverse / Jensen-Shannon self-distillation divergence and the teacher an EMA of the
  student's weights (steps.rs:3502-3554); the mask keeps all tokens, the supervised
  (target) tokens or the unsupervised (context) ones.

Every weight is 0 before ``warmup_steps``, ramps linearly over ``ramp_steps`` and is
active only on steps that are multiples of ``every_steps``, so the trainer runs its
fused CE step on every step where all weights are 0.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..config import DynamicsAnchorConfig, LogitEntropyFloorConfig, RepeatUnlikelihoodConfig

_EPS = 1.1920929e-07  # f32 machine epsilon, the reference's "weight is off" threshold


def scheduled_weight(enabled: bool, weight: float, warmup: int, ramp: int, every: int, step: int) -> float:
    if every > 1 and step % every != 0:
        return 0.0
    if not enabled or weight <= _EPS or step < warmup:
        return 0.0
    if ramp == 0:
        return weight
    return weight * min(max((step - warmup + 1) / ramp, 0.0), 1.0)


def _w(cfg, weight: float, step: int) -> float:
    return scheduled_weight(cfg.enabled, weight, cfg.warmup_steps, cfg.ramp_steps, cfg.every_steps, step)


def entropy_floor_loss(log_probs: torch.Tensor, targets: torch.Tensor, cfg: LogitEntropyFloorConfig,
                       step: int) -> torch.Tensor | None:
    V = log_probs.shape[-1]
    lp = log_probs.reshape(-1, V)
    if lp.shape[0] == 0 or V == 0:
        return None
    p = lp.exp()
    w, wm, wc = _w(cfg, cfg.weight, step), _w(cfg, cfg.marginal_weight, step), _w(cfg, cfg.target_coverage_weight, step)
    total = None

    def add(t):
        nonlocal total
        total = t if total is None else total + t

    if w > _EPS and cfg.target_entropy_bits > _EPS:
        ent = -(p * lp).sum(1).mean()
        add(w * (cfg.target_entropy_bits * math.log(2.0) - ent).clamp_min(0.0))
    if wm > _EPS or wc > _EPS:
        marg = p.mean(0)
        if wm > _EPS and cfg.target_marginal_entropy_bits > _EPS:
            ent = -(marg * marg.clamp_min(1e-12).log()).sum()
            add(wm * (cfg.target_marginal_entropy_bits * math.log(2.0) - ent).clamp_min(0.0))
        if wc > _EPS and 0.0 < cfg.target_coverage_epsilon < 1.0:
            add(-wc * marg.clamp_min(cfg.target_coverage_epsilon).log()[targets.reshape(-1)].mean())
    return total


def _unlikelihood(lp_sel: torch.Tensor, eps: float) -> torch.Tensor:
    return -(1.0 - lp_sel.exp().clamp(0.0, 1.0 - eps)).clamp_min(eps).log()


def repeat_lags(cfg: RepeatUnlikelihoodConfig, T: int) -> list[int]:
    return sorted({lag for lag in [1, *cfg.history_lags] if 1 <= lag <= T}) if T else []


def cycle_lags(cfg: RepeatUnlikelihoodConfig, T: int, step: int) -> list[int]:
    if T == 0 or cfg.cycle_min_lag == 0 or cfg.cycle_max_lag < cfg.cycle_min_lag:
        return []
    lo, hi = min(cfg.cycle_min_lag, T), min(cfg.cycle_max_lag, T)
    if hi < lo:
        return []
    avail = hi - lo + 1
    budget = min(max(cfg.cycle_lags_per_step, 1), avail)
    if budget == avail:
        return list(range(lo, hi + 1))
    stride = max(avail // budget, 1)
    off = step % avail
    return sorted({lo + (off + i * stride) % avail for i in range(budget)})


def _lagged(log_probs, targets, inputs, lag):
    s = lag - 1
    T = log_probs.shape[1]
    return log_probs[:, s:], targets[:, s:], inputs[:, :T - s]


def repeat_unlikelihood_loss(logits, log_probs, targets, inputs, cfg: RepeatUnlikelihoodConfig,
                             step: int) -> torch.Tensor | None:
    T = log_probs.shape[1]
    w, wc, wm = _w(cfg, cfg.weight, step), _w(cfg, cfg.cycle_weight, step), _w(cfg, cfg.cycle_margin_weight, step)
    total = None

    def add(t):
        nonlocal total
        total = t if total is None else total + t

    if w > _EPS:
        num, hits = 0.0, 0.0
        for lag in repeat_lags(cfg, T):
            lp, tg, hist = _lagged(log_probs, targets, inputs, lag)
            m = (hist != tg).to(lp.dtype)
            num = num + (_unlikelihood(lp.gather(-1, hist.unsqueeze(-1)).squeeze(-1), cfg.epsilon) * m).sum()
            hits = hits + m.sum()
        if not isinstance(num, float):
            add(w * num / hits.clamp_min(1.0))
    if wc > _EPS or wm > _EPS:
        mean_logits = logits.float().mean(-1) if wm > _EPS else None
        cn, ch, mn, mh = 0.0, 0.0, 0.0, 0.0
        for lag in cycle_lags(cfg, T, step):
            lp, tg, hist = _lagged(log_probs, targets, inputs, lag)
            m = (hist != tg).to(lp.dtype)
            if wc > _EPS:
                cn = cn + (_unlikelihood(lp.gather(-1, hist.unsqueeze(-1)).squeeze(-1), cfg.epsilon) * m).sum()
                ch = ch + m.sum()
            if wm > _EPS:
                s = lag - 1
                hl = logits[:, s:].float().gather(-1, hist.unsqueeze(-1)).squeeze(-1)
                mn = mn + (F.softplus(hl - mean_logits[:, s:] + cfg.cycle_margin) * m).sum()
                mh = mh + m.sum()
        if not isinstance(cn, float):
            add(wc * cn / ch.clamp_min(1.0))
        if not isinstance(mn, float):
            add(wm * mn / mh.clamp_min(1.0))
    return total


def anchor_mask(cfg: DynamicsAnchorConfig, loss_mask):
    if cfg.mask == "all_tokens" or loss_mask is None:
        return None
    return loss_mask if cfg.mask == "target_tokens" else (loss_mask == 0)


def dynamics_anchor_loss(student_lp, teacher_logits, cfg: DynamicsAnchorConfig, step: int,
                         loss_mask=None) -> torch.Tensor | None:
    from .objectives import masked_token_mean, self_distillation_per_token

    w = _w(cfg, cfg.weight, step)
    if w <= _EPS:
        return None
    per = self_distillation_per_token(student_lp, F.log_softmax(teacher_logits.detach().float(), -1), cfg.kl)
    return w * masked_token_mean(per, anchor_mask(cfg, loss_mask))


class LogitRegularizers:
    """The configured auxiliary terms of one training run."""

    def __init__(self, entropy: LogitEntropyFloorConfig, repeat: RepeatUnlikelihoodConfig,
                 anchor: DynamicsAnchorConfig | None = None):
        self.entropy, self.repeat = entropy, repeat
        self.anchor = anchor or DynamicsAnchorConfig()

    def enabled(self) -> bool:
        return self.entropy.enabled or self.repeat.enabled or self.anchor.enabled

    def anchor_active(self, step: int) -> bool:
        return _w(self.anchor, self.anchor.weight, step) > _EPS

    def active(self, step: int) -> bool:
        e, r = self.entropy, self.repeat
        return self.anchor_active(step) or any(
            x > _EPS for x in (_w(e, e.weight, step), _w(e, e.marginal_weight, step),
                               _w(e, e.target_coverage_weight, step), _w(r, r.weight, step),
                               _w(r, r.cycle_weight, step), _w(r, r.cycle_margin_weight, step)))

    def loss(self, logits, targets, inputs, step: int, mask=None, teacher_logits=None) -> torch.Tensor:
        """Next-token CE plus the active auxiliary terms."""
        lp = F.log_softmax(logits.float(), -1)
        nll = -lp.gather(-1, targets.unsqueeze(-1)).squeeze(-1)
        if mask is None:
            loss = nll.mean()
        else:
            mk = mask.to(nll.dtype)
            loss = (nll * mk).sum() / mk.sum().clamp_min(1.0)
        terms = [repeat_unlikelihood_loss(logits, lp, targets, inputs, self.repeat, step),
                 entropy_floor_loss(lp, targets, self.entropy, step)]
        if teacher_logits is not None:
            terms.append(dynamics_anchor_loss(lp, teacher_logits, self.anchor, step, mask))
        for aux in terms:
            if aux is not None:
                loss = loss + aux
        return loss

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

* greedy rollout unlikelihood (steps.rs:10684-11067, prompt placement :13029-13046):
  every ``every_steps`` steps a prompt window of the clean inputs is run through the
  model with recurrent state and continued greedily for ``rollout_tokens`` tokens,
  backpropagating through the rollout; each greedy token that repeats one of the last
  ``history_tokens`` tokens is pushed down (unlikelihood, and a softplus margin over
  the mean logit), the same on the cycle lags, the rollout's per-step entropy is
  floored, and ``recovery`` / ``sequence_recovery`` score the true continuation one
  step at a time or with one teacher-forced pass over prompt + rollout.

Every weight is 0 before ``warmup_steps``, ramps linearly over ``ramp_steps`` and is
active only on steps that are multiples of ``every_steps``, so the trainer runs its
fused CE step on every step where all weights are 0.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..config import (DynamicsAnchorConfig, GreedyRolloutUnlikelihoodConfig, LogitEntropyFloorConfig,
                      RepeatUnlikelihoodConfig)

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


def rollout_prompt_start(step: int, every: int, block: int, prompt: int) -> int:
    avail = max(block - prompt, 0)
    if avail == 0:
        return 0
    lo = min(avail, max(prompt, 1))
    span = avail - lo
    if span == 0:
        return lo
    return lo + ((step // max(every, 1)) * max(prompt, 1)) % (span + 1)


def _ramped(cfg, weight: float, step: int) -> float:
    # the rollout's terms ramp like the others; its cadence gates the whole rollout
    return scheduled_weight(cfg.enabled, weight, cfg.warmup_steps, cfg.ramp_steps, 1, step)


def greedy_rollout_active(cfg: GreedyRolloutUnlikelihoodConfig, step: int) -> bool:
    if not cfg.enabled or cfg.recovery_only or step % max(cfg.every_steps, 1) != 0:
        return False
    return any(_ramped(cfg, w, step) > _EPS for w in (
        cfg.weight, cfg.margin_weight, cfg.cycle_weight, cfg.cycle_margin_weight, cfg.recovery_weight,
        cfg.sequence_recovery_weight, cfg.entropy_floor_weight))


def greedy_rollout_loss(model, clean_inputs: torch.Tensor, cfg: GreedyRolloutUnlikelihoodConfig,
                        step: int) -> torch.Tensor | None:
    """``model(tokens, state=ModelState)`` -> logits; the state carries rho between calls."""
    from ..models.state import ModelState

    if not greedy_rollout_active(cfg, step):
        return None
    w, wm = _ramped(cfg, cfg.weight, step), _ramped(cfg, cfg.margin_weight, step)
    wc, wcm = _ramped(cfg, cfg.cycle_weight, step), _ramped(cfg, cfg.cycle_margin_weight, step)
    wr, wsr = _ramped(cfg, cfg.recovery_weight, step), _ramped(cfg, cfg.sequence_recovery_weight, step)
    we = _ramped(cfg, cfg.entropy_floor_weight, step)
    B, T = clean_inputs.shape
    pb, pt = min(B, max(cfg.batch_prompts, 1)), min(T, max(cfg.prompt_tokens, 1))
    p0 = rollout_prompt_start(step, cfg.every_steps, T, pt)
    prompt = clean_inputs[:pb, p0:p0 + pt]
    need_grad = any(x > _EPS for x in (w, wm, wc, wcm, wr, we))
    state = ModelState.empty()
    with torch.set_grad_enabled(need_grad and torch.is_grad_enabled()):
        last = model(prompt, state=state)[:, -1].float()
        hist_n = max(cfg.history_tokens, 1)
        history = [prompt[:, pt - 1 - o] for o in range(min(pt, hist_n))]  # newest first
        sums = {k: [None, None] for k in ("u", "m", "c", "cm")}
        rec, rec_n, ent, ent_n, generated = None, 0, None, 0, []

        def acc(key, value, mask):
            m = mask.to(value.dtype)
            v, h = (value * m).sum(), m.sum()
            a = sums[key]
            sums[key] = [v if a[0] is None else a[0] + v, h if a[1] is None else a[1] + h]

        for r in range(cfg.rollout_tokens):
            lp = F.log_softmax(last, -1)
            if we > _EPS and cfg.target_entropy_bits > _EPS:
                e = (cfg.target_entropy_bits * math.log(2.0) + (lp.exp() * lp).sum(-1).mean()).clamp_min(0.0) * we
                ent, ent_n = (e if ent is None else ent + e), ent_n + 1
            nxt = last.argmax(-1)
            rep = torch.zeros_like(nxt, dtype=torch.bool)
            for h in history:
                rep |= nxt == h
            cyc = None
            if cfg.cycle_min_lag > 0 and cfg.cycle_max_lag >= cfg.cycle_min_lag:
                for lag in range(cfg.cycle_min_lag, cfg.cycle_max_lag + 1):
                    if lag - 1 < len(history):
                        hit = nxt == history[lag - 1]
                        cyc = hit if cyc is None else cyc | hit
            sel = lp.gather(-1, nxt[:, None]).squeeze(-1)
            margin = F.softplus(last.gather(-1, nxt[:, None]).squeeze(-1) - last.mean(-1) + cfg.margin)
            if w > _EPS:
                acc("u", _unlikelihood(sel, cfg.epsilon), rep)
            if wc > _EPS and cyc is not None:
                acc("c", _unlikelihood(sel, cfg.epsilon), cyc)
            if wm > _EPS:
                acc("m", margin, rep)
            if wcm > _EPS and cyc is not None:
                acc("cm", margin, cyc)
            tpos = p0 + pt + r
            if wr > _EPS and tpos < T:
                nll = -lp.gather(-1, clean_inputs[:pb, tpos:tpos + 1]).squeeze(-1).mean()
                rec, rec_n = (nll if rec is None else rec + nll), rec_n + 1
            generated.append(nxt)
            last = model(nxt[:, None], state=state)[:, -1].float()
            history.insert(0, nxt)
            del history[hist_n:]
    total = None

    def add(t):
        nonlocal total
        total = t if total is None else total + t

    for key, wt in (("u", w), ("m", wm), ("c", wc), ("cm", wcm)):
        v, h = sums[key]
        if v is not None:
            add(wt * v / h.clamp_min(1.0))
    if rec is not None and rec_n:
        add(rec * (wr / rec_n))
    if wsr > _EPS and generated and p0 + pt < T:
        n = min(len(generated), T - p0 - pt)
        seq = torch.cat([prompt, torch.stack(generated[:n], 1)], 1)
        lg = model(seq)[:, pt - 1:pt - 1 + n].float()
        tg = clean_inputs[:pb, p0 + pt:p0 + pt + n]
        add(wsr * -F.log_softmax(lg, -1).gather(-1, tg.unsqueeze(-1)).mean())
    if ent is not None and ent_n:
        add(ent / ent_n)
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
                 anchor: DynamicsAnchorConfig | None = None, rollout: GreedyRolloutUnlikelihoodConfig | None = None):
        self.entropy, self.repeat = entropy, repeat
        self.anchor = anchor or DynamicsAnchorConfig()
        self.rollout = rollout or GreedyRolloutUnlikelihoodConfig()

    def enabled(self) -> bool:
        return self.entropy.enabled or self.repeat.enabled or self.anchor.enabled or self.rollout.enabled

    def anchor_active(self, step: int) -> bool:
        return _w(self.anchor, self.anchor.weight, step) > _EPS

    def active(self, step: int) -> bool:
        e, r = self.entropy, self.repeat
        return self.anchor_active(step) or greedy_rollout_active(self.rollout, step) or any(
            x > _EPS for x in (_w(e, e.weight, step), _w(e, e.marginal_weight, step),
                               _w(e, e.target_coverage_weight, step), _w(r, r.weight, step),
                               _w(r, r.cycle_weight, step), _w(r, r.cycle_margin_weight, step)))

    def loss(self, logits, targets, inputs, step: int, mask=None, teacher_logits=None, model=None,
             clean_inputs=None) -> torch.Tensor:
        """Next-token CE plus the active auxiliary terms (the greedy rollout needs
        ``model`` and the uncorrupted inputs)."""
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
        if model is not None:
            terms.append(greedy_rollout_loss(model, inputs if clean_inputs is None else clean_inputs,
                                             self.rollout, step))
        for aux in terms:
            if aux is not None:
                loss = loss + aux
        return loss

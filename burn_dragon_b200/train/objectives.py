"""Training objectives: next-token CE and the self-distillation family (SDFT / SDPO).

Reference: burn_dragon_core/src/objective.rs. Pieces:

* KL kinds per token: ``forward`` KL(teacher || student), ``reverse`` KL(student ||
  teacher), ``jensen_shannon`` (mean of both KLs to the mixture, probabilities clamped
  at 1e-12 before the log) (objective.rs:528-552, 802-810);
* ``masked_token_mean`` (objective.rs:812-824);
* SDPO token advantage (teacher - student selected-token log-prob, optionally
  normalised over the batch) and the PPO-style clipped policy loss (objective.rs:566-627);
* selected-token log-prob MSE distillation (objective.rs:628-695);
* window objectives on a token window: ``sdft`` = selected-token MSE between student and
  teacher log-probs of the targets, ``sdpo`` = the same with the KL kind chosen from
  ``alpha`` (reverse for alpha >= 1 squares teacher - student), ``sdft_sdpo`` = the
  normalised weighted sum (objective.rs:696-760);
* the teacher is an EMA of the student (``teacher_update_rate``).

Configs keep the reference's field names and validation rules (objective.rs:116-424).
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F


@dataclass
class SdftObjectiveConfig:
    max_completion_tokens: int = 32
    temperature: float = 1.0
    top_k: int | None = None
    kl: str = "forward"  # forward | reverse | jensen_shannon
    generate_from_teacher: bool = False
    teacher_update_rate: float = 0.01
    top_entropy_quantile: float | None = None
    num_loss_tokens_to_skip: int = 0

    def validate(self, path: str = "training.objective") -> None:
        if self.max_completion_tokens <= 0:
            raise ValueError(f"{path}.max_completion_tokens must be > 0")
        if not self.temperature > 0:
            raise ValueError(f"{path}.temperature must be > 0")
        if self.top_k is not None and self.top_k <= 0:
            raise ValueError(f"{path}.top_k must be > 0 when set")
        if not 0.0 <= self.teacher_update_rate <= 1.0:
            raise ValueError(f"{path}.teacher_update_rate must be in [0, 1]")
        if self.top_entropy_quantile is not None:
            raise ValueError(f"{path}.top_entropy_quantile is not wired into rollout masking")


@dataclass
class SdpoObjectiveConfig:
    group_size: int = 2
    max_completion_tokens: int = 32
    temperature: float = 1.0
    top_k: int | None = None
    full_logit_distillation: bool = True
    alpha: float = 0.5
    success_reward_threshold: float = 0.0
    teacher_regularization: str = "ema"
    teacher_update_rate: float = 0.05
    distillation_topk: int | None = None
    distillation_add_tail: bool = False
    is_clip: float | None = 2.0

    def kl_kind(self) -> str:
        return "forward" if self.alpha <= 0 else "reverse" if self.alpha >= 1 else "jensen_shannon"

    def validate(self, path: str = "training.objective") -> None:
        if self.group_size <= 0 or self.max_completion_tokens <= 0:
            raise ValueError(f"{path}.group_size and max_completion_tokens must be > 0")
        if not 0.0 <= self.alpha <= 1.0:
            raise ValueError(f"{path}.alpha must be in [0, 1]")
        if self.success_reward_threshold > 0:
            raise ValueError(f"{path}.success_reward_threshold needs an external reward source")
        if not self.full_logit_distillation:
            raise ValueError(f"{path}.full_logit_distillation=false is not supported")
        if self.teacher_regularization != "ema":
            raise ValueError(f"{path}.teacher_regularization supports only \"ema\"")


@dataclass
class ObjectiveConfig:
    type: str = "next_token"  # next_token | sdft | sdpo | sdft_sdpo
    sdft: SdftObjectiveConfig = field(default_factory=SdftObjectiveConfig)
    sdpo: SdpoObjectiveConfig = field(default_factory=SdpoObjectiveConfig)
    sdft_weight: float = 0.5
    sdpo_weight: float = 0.5

    def validate(self) -> None:
        if self.type not in ("next_token", "sdft", "sdpo", "sdft_sdpo"):
            raise ValueError(f"unknown objective {self.type!r}")
        if self.type in ("sdft", "sdft_sdpo"):
            self.sdft.validate()
        if self.type in ("sdpo", "sdft_sdpo"):
            self.sdpo.validate()
        if self.type == "sdft_sdpo" and not (self.sdft_weight > 0 and self.sdpo_weight > 0):
            raise ValueError("training.objective weights must be > 0")


def masked_token_mean(values: torch.Tensor, mask: torch.Tensor | None = None) -> torch.Tensor:
    if mask is None:
        return values.mean()
    m = mask.to(values.dtype)
    return (values * m).sum() / m.sum().clamp_min(1.0)


def _kl(left_lp: torch.Tensor, right_lp: torch.Tensor) -> torch.Tensor:
    return (left_lp.exp() * (left_lp - right_lp)).sum(-1)


def self_distillation_per_token(student_lp, teacher_lp, kind: str) -> torch.Tensor:
    if kind == "forward":
        return _kl(teacher_lp, student_lp)
    if kind == "reverse":
        return _kl(student_lp, teacher_lp)
    mix = (0.5 * (student_lp.exp() + teacher_lp.exp())).clamp_min(1e-12).log()
    return 0.5 * (_kl(teacher_lp, mix) + _kl(student_lp, mix))


def self_distillation_loss_from_logits(student_logits, teacher_logits, mask=None, kind: str = "forward"):
    return masked_token_mean(self_distillation_per_token(F.log_softmax(student_logits.float(), -1),
                                                         F.log_softmax(teacher_logits.float(), -1), kind), mask)


def selected_token_log_probs(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    return F.log_softmax(logits.float(), -1).gather(-1, targets.unsqueeze(-1)).squeeze(-1)


def sdpo_token_advantage(teacher_lp, student_lp, mask=None, normalize: bool = False, eps: float = 1e-6):
    adv = teacher_lp - student_lp
    if mask is not None:
        adv = adv * mask.to(adv.dtype)
    if not normalize:
        return adv
    c = adv - adv.mean()
    return c / (c.pow(2).mean() + max(eps, 1e-12)).sqrt()


def clipped_policy_loss(lp_new, lp_old, advantage, mask=None, clip: float | None = None, weight: float = 1.0):
    weight = max(weight, 0.0)
    if weight <= 0:
        return lp_new.new_zeros(())
    if clip is not None and clip > 0:
        ratio = (lp_new - lp_old).clamp(-20.0, 20.0).exp()
        obj = torch.minimum(ratio * advantage, ratio.clamp(1 - clip, 1 + clip) * advantage)
    else:
        obj = lp_new * advantage
    return masked_token_mean(-weight * obj, mask)


def selected_token_log_prob_mse(student_lp, teacher_lp, mask=None):
    return masked_token_mean((student_lp - teacher_lp.detach()).pow(2), mask)


def window_objective_loss(student, teacher, inputs, targets, cfg: ObjectiveConfig, mask=None):
    """Loss of one token window; ``student`` / ``teacher`` map tokens to logits."""
    if cfg.type == "next_token":
        lg = student(inputs)
        return masked_token_mean(-selected_token_log_probs(lg, targets), mask)
    s_lp = selected_token_log_probs(student(inputs), targets)
    with torch.no_grad():
        t_lp = selected_token_log_probs(teacher(inputs), targets)

    def sdpo():
        if cfg.sdpo.kl_kind() == "reverse":
            return masked_token_mean((t_lp - s_lp).pow(2), mask)
        return selected_token_log_prob_mse(s_lp, t_lp, mask)

    if cfg.type == "sdft":
        return selected_token_log_prob_mse(s_lp, t_lp, mask)
    if cfg.type == "sdpo":
        return sdpo()
    ws, wp = max(cfg.sdft_weight, 0.0), max(cfg.sdpo_weight, 0.0)
    tot = max(ws + wp, 1e-6)
    return selected_token_log_prob_mse(s_lp, t_lp, mask) * (ws / tot) + sdpo() * (wp / tot)


class EMATeacher:
    """Teacher = exponential moving average of the student's parameters."""

    def __init__(self, student: torch.nn.Module, rate: float):
        self.rate = rate
        self.model = copy.deepcopy(student)
        for p in self.model.parameters():
            p.requires_grad_(False)

    @torch.no_grad()
    def update(self, student: torch.nn.Module) -> None:
        for t, s in zip(self.model.parameters(), student.parameters()):
            t.lerp_(s.detach(), self.rate)

"""Per-module learning-rate scales, optionally scheduled.

Reference: ``module_lr_scales`` entries {target, scale, schedule {final_scale,
start_fraction, end_fraction}} (burn_dragon_language/src/config/train/schema.rs:
133-150) with the schedule rule of burn_dragon_language/src/train/steps.rs:53-107: the
scale is ``scale`` up to step round(start_fraction * (total - 1)), ``final_scale`` from
step round(end_fraction * (total - 1)), linear in between.

Targets of the BDH parameter store: ``embedding`` (embed), ``normalization`` (norm_*),
``output_head`` (lm_head), ``shared_lowrank_encoder`` (encoder, encoder_v),
``shared_lowrank_decoder`` (decoder). The scale multiplies the AdamW update of those
tensors (update = new - old after the fused optimizer step), which is a learning-rate
multiplier including the decoupled weight decay.
"""

from __future__ import annotations

import torch

TARGETS = {
    "embedding": ("embed",),
    "normalization": ("norm_gamma", "norm_beta", "norm_alpha", "norm_shift"),
    "output_head": ("lm_head",),
    "shared_lowrank_encoder": ("encoder", "encoder_v"),
    "shared_lowrank_decoder": ("decoder",),
}


class ScaleRule:
    def __init__(self, scale: float, schedule: dict | None, total_steps: int):
        self.initial = float(scale)
        self.final = float(scale)
        self.start = self.end = 0
        if schedule:
            last = max(total_steps, 1) - 1
            self.final = float(schedule["final_scale"])
            self.start = round(last * min(max(float(schedule.get("start_fraction", 0.0)), 0.0), 1.0))
            self.end = round(last * min(max(float(schedule.get("end_fraction", 1.0)), 0.0), 1.0))

    def at(self, step: int) -> float:
        if step <= self.start:
            return self.initial
        if step >= self.end or self.end <= self.start:
            return self.final
        return self.initial + (self.final - self.initial) * (step - self.start) / (self.end - self.start)


class ModuleLrScales:
    def __init__(self, entries: list[dict], total_steps: int):
        self.rules: list[tuple[tuple[str, ...], ScaleRule]] = []
        for e in entries:
            t = e["target"]
            if t not in TARGETS:
                raise ValueError(f"module_lr_scales: target {t!r} is not a parameter-store module "
                                 f"({sorted(TARGETS)})")
            self.rules.append((TARGETS[t], ScaleRule(e.get("scale", 1.0), e.get("schedule"), total_steps)))
        self._before: dict[str, torch.Tensor] | None = None

    def before_step(self, model, step: int) -> None:
        self._before = {}
        for names, rule in self.rules:
            if rule.at(step) != 1.0:
                for n in names:
                    if n in model.store.shapes:
                        self._before[n] = getattr(model, n).detach().clone()
        self._model = model

    @torch.no_grad()
    def after_step(self, step: int) -> None:
        if not self._before:
            return
        m = self._model
        for names, rule in self.rules:
            s = rule.at(step)
            for n in names:
                if n in self._before:
                    p = getattr(m, n)
                    b = self._before[n]
                    p.copy_(b + (p - b) * s)
        m.store.refresh_shadow()
        self._before = None

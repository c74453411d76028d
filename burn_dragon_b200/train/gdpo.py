"""GDPO advantage gating (burn_dragon_train/src/train/gdpo/mod.rs:30-415): rewards of a
group of samples per prompt are normalised per group, and a per-row percentile threshold
gates which samples keep a positive advantage. ``percentile_thresholds`` runs the CUDA
kernel on GPU tensors and the same interpolation rule in PyTorch otherwise.
"""

from __future__ import annotations

import torch

from .. import _ext


def percentile_thresholds_ref(values: torch.Tensor, q: float) -> torch.Tensor:
    v = torch.nan_to_num(values.float(), nan=0.0, posinf=torch.finfo(torch.float32).max,
                         neginf=-torch.finfo(torch.float32).max)
    s, _ = torch.sort(v, dim=1)
    g = s.shape[1]
    pos = (g - 1) * q
    lo = int(pos)
    hi = min(lo + 1, g - 1)
    w = pos - lo
    return s[:, lo] + (s[:, hi] - s[:, lo]) * w


def percentile_thresholds(values: torch.Tensor, q: float) -> torch.Tensor:
    if values.is_cuda:
        out = torch.empty(values.shape[0], device=values.device)
        _ext.load().percentile_thresholds(values.float().contiguous(), float(q), out)
        return out
    return percentile_thresholds_ref(values, q)


def gdpo_advantages(rewards: torch.Tensor, quantile: float = 0.5, eps: float = 1e-6) -> torch.Tensor:
    """rewards [prompts, group] -> advantages: group-normalised rewards, zeroed for
    samples below the group's ``quantile`` threshold."""
    mean = rewards.mean(1, keepdim=True)
    std = rewards.std(1, keepdim=True, unbiased=False)
    adv = (rewards - mean) / (std + eps)
    thr = percentile_thresholds(rewards, quantile)
    return torch.where(rewards >= thr[:, None], adv, torch.zeros_like(adv))

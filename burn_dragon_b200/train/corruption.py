"""Causal input corruption: each input token is replaced, with the scheduled probability,
by ``replacement_token_id`` or a uniform random token (burn_dragon_language/src/train/
steps.rs:11070-11095). Targets are untouched, so the model learns to predict the clean
next token from a noisy prefix. Applied on the host batch before its device copy, from a
generator seeded by (seed, step, rank) so runs and resumes are reproducible."""

from __future__ import annotations

import torch

from ..config import CausalInputCorruptionConfig


def corrupt_inputs(x: torch.Tensor, cfg: CausalInputCorruptionConfig, step: int, vocab: int, seed: int = 0,
                   rank: int = 0) -> torch.Tensor:
    p = cfg.probability_at(step)
    if p <= 0.0:
        return x
    g = torch.Generator().manual_seed((seed * 1_000_003 + step) * 65_537 + rank)
    mask = torch.rand(x.shape, generator=g) < p
    if cfg.replacement_token_id is not None:
        rep = torch.full(x.shape, int(cfg.replacement_token_id), dtype=x.dtype)
    else:
        rep = torch.randint(0, max(vocab, 1), x.shape, generator=g, dtype=x.dtype)
    return torch.where(mask, rep, x.cpu()).to(x.device)

"""EGGROLL: evolution strategies with antithetic low-rank perturbations of the matrix
parameters, the whole population evaluated in one batched forward
(burn_dragon_eggroll/src/lib.rs:96-238; population forward dragon.rs:1555-1646).

Member i of a population of 2P uses ``W + s_i * sigma * A_i B_i^T / sqrt(r)`` with
s_i = +-1 (antithetic pairs share A_i, B_i), A_i, B_i Gaussian of rank r, for the three
shared projections. Fitness is minus the CE loss on the batch; the update is
``W += lr / (2 P sigma) * sum_i (f_i^+ - f_i^-) E_i`` (the antithetic ES estimator).
All members run in one forward: the population is a leading batch dimension of the
weights (``torch.func.vmap`` over members).
"""

from __future__ import annotations

import math

import torch

from ..models import reference as R

MATRIX = ("encoder", "encoder_v", "decoder")


def _noise(shape, rank: int, gen: torch.Generator, device):
    if len(shape) == 3:
        H, a, b = shape
        A = torch.randn(H, a, rank, generator=gen).to(device)
        B = torch.randn(H, rank, b, generator=gen).to(device)
    else:
        a, b = shape
        A = torch.randn(a, rank, generator=gen).to(device)
        B = torch.randn(rank, b, generator=gen).to(device)
    return torch.matmul(A, B) / math.sqrt(rank)


@torch.no_grad()
def population_losses(model, tokens, targets, noises: dict, sigma: float) -> torch.Tensor:
    """Losses of the 2P antithetic members (order: +1..+P, -1..-P), one batched forward."""
    base = model.param_dict()
    cfg = model.cfg
    P = next(iter(noises.values())).shape[0]

    def member_loss(sign, *eps):
        p = dict(base)
        for n, e in zip(MATRIX, eps):
            p[n] = base[n] + sign * sigma * e
        logits, _ = R.bdh_forward(tokens, p, cfg)
        return R.cross_entropy(logits, targets)

    signs = torch.cat([torch.ones(P), -torch.ones(P)]).to(tokens.device)
    eps = [torch.cat([noises[n], noises[n]], 0) for n in MATRIX]
    return torch.func.vmap(member_loss)(signs, *eps)


@torch.no_grad()
def normalize_fitness(f: torch.Tensor, kind: str) -> torch.Tensor:
    """``none``; ``center`` (minus the population mean); ``rank``: centred ranks in
    [-0.5, 0.5] (the usual ES rank transform; ties broken by order). The reference names
    these modes (burn_dragon_eggroll/src/lib.rs:139-175) but defines them in the
    ``burn_eggroll`` crate, which is not in its repository, so these are the standard forms."""
    if kind == "none":
        return f
    if kind == "center":
        return f - f.mean()
    if kind == "rank":
        n = f.numel()
        r = torch.empty_like(f)
        r[torch.argsort(f)] = torch.arange(n, dtype=f.dtype, device=f.device)
        return r / max(n - 1, 1) - 0.5
    raise ValueError(f"unknown fitness normalization {kind!r}")


@torch.no_grad()
def es_step(model, tokens, targets, population: int = 8, sigma: float = 0.01, lr: float = 0.01, rank: int = 4,
            seed: int = 0, chunk: int | None = None, weight_decay: float = 0.0, reduce=None,
            fitness_normalization: str = "none", coefficient_clip: float | None = None,
            max_delta_rms: float | None = None) -> dict:
    """One antithetic ES update of the three shared projections; returns diagnostics.

    ``population`` antithetic pairs (2 x population members), evaluated ``chunk`` pairs
    per batched forward; ``weight_decay`` is decoupled (W *= 1 - lr * wd before the ES
    step); ``reduce`` maps this rank's member losses to the data-parallel mean, so every
    rank (same ``seed``, hence the same perturbations) applies the same update.
    ``fitness_normalization`` transforms the 2P fitnesses before the pair coefficients,
    ``coefficient_clip`` clamps each pair's coefficient and ``max_delta_rms`` rescales a
    matrix's update so its RMS stays under that bound."""
    gen = torch.Generator().manual_seed(seed)
    params = model.param_dict()
    noises = {n: torch.stack([_noise(params[n].shape, rank, gen, tokens.device) for _ in range(population)])
              for n in MATRIX}
    step = max(1, min(chunk or population, population))
    plus, minus = [], []
    for c in range(0, population, step):
        part = population_losses(model, tokens, targets, {n: noises[n][c:c + step] for n in MATRIX}, sigma)
        k = part.shape[0] // 2
        plus.append(part[:k])
        minus.append(part[k:])
    losses = torch.cat(plus + minus)
    if reduce is not None:
        losses = reduce(losses)
    fit = normalize_fitness(-losses, fitness_normalization)
    fp, fm = fit[:population], fit[population:]
    coef = (fp - fm) / (2 * population * sigma)
    if coefficient_clip is not None:
        coef = coef.clamp(-coefficient_clip, coefficient_clip)
    for n in MATRIX:
        w = getattr(model, n)
        if weight_decay:
            w.mul_(1.0 - lr * weight_decay)
        upd = lr * torch.tensordot(coef, noises[n], dims=1)
        if max_delta_rms is not None:
            rms = float(upd.pow(2).mean().sqrt())
            if rms > max_delta_rms:
                upd = upd * (max_delta_rms / rms)
        w.add_(upd)
    model.store.refresh_shadow()
    return {"mean_loss": float(losses.mean()), "best_loss": float(losses.min())}


def es_gradient_estimate(model, tokens, targets, population: int, sigma: float, rank: int, seed: int = 0) -> dict:
    """The ES estimate of -dL/dW (for diagnostics / tests)."""
    gen = torch.Generator().manual_seed(seed)
    params = model.param_dict()
    noises = {n: torch.stack([_noise(params[n].shape, rank, gen, tokens.device) for _ in range(population)])
              for n in MATRIX}
    losses = population_losses(model, tokens, targets, noises, sigma)
    coef = (-losses[:population] + losses[population:]) / (2 * population * sigma)
    return {n: torch.tensordot(coef, noises[n], dims=1) for n in MATRIX}

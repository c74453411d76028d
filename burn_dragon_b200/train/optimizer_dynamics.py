"""Optimizer-dynamics comparison: the same model, data and number of steps trained with
AdamW and with EGGROLL, reporting initial / final train and held-out losses, wall time,
forward evaluations and the derived rates (burn_dragon_language/src/train/
optimizer_dynamics.rs:25-160, defaults :47-66). Runs through the PyTorch path; a
diagnostic, not a training path.
"""

from __future__ import annotations

import time
from dataclasses import asdict, dataclass

import torch

from ..models import reference as R
from .eggroll import es_step
from .optim import FusedAdamW


@dataclass
class OptimizerDynamicsConfig:
    max_iters: int = 512
    seed: int = 29
    adamw_learning_rate: float = 2.5e-2
    eggroll_learning_rate: float = 1.0e-1
    eggroll_sigma: float = 1.0e-2
    eggroll_interval_steps: int = 1
    eggroll_population_size: int = 256
    eggroll_rank: int = 4
    eggroll_coefficient_clip: float | None = 128.0
    eggroll_fitness_normalization: str = "rank"
    eggroll_max_delta_rms: float | None = 1.0e-1


def _loss(model, x, y) -> float:
    with torch.no_grad():
        return float(R.cross_entropy(model(x), y))


def run_optimizer_dynamics(kind: str, make_model, batches, held, cfg: OptimizerDynamicsConfig) -> dict:
    """``make_model``: a callable returning a fresh model (the same initial weights for
    each arm; the flat parameter store is not deep-copied); ``batches``: a callable
    step -> (x, y); ``held``: a fixed (x, y) for the held-out loss."""
    m = make_model()
    x0, y0 = batches(0)
    r = {"optimizer": kind, "seed": cfg.seed, "initial_train_loss": _loss(m, x0, y0),
         "initial_loss": _loss(m, *held)}
    evals, steps = 0, 0
    opt = FusedAdamW(m.store, lr=cfg.adamw_learning_rate, weight_decay=0.0) if kind == "adamw" else None
    t0 = time.perf_counter()
    for i in range(cfg.max_iters):
        x, y = batches(i)
        if kind == "adamw":
            loss = R.cross_entropy(m(x), y)
            grads = torch.autograd.grad(loss, list(m.parameters()), allow_unused=True)
            for (n, _), g in zip(m.named_parameters(), grads):
                view = m.store.view(m.store.grad, n)
                view.zero_() if g is None else view.copy_(g)
            opt.step()
            evals += 1
        elif i % max(cfg.eggroll_interval_steps, 1) == 0:
            es_step(m, x, y, population=cfg.eggroll_population_size // 2, sigma=cfg.eggroll_sigma,
                    lr=cfg.eggroll_learning_rate, rank=cfg.eggroll_rank, seed=cfg.seed * 1_000_003 + i,
                    fitness_normalization=cfg.eggroll_fitness_normalization,
                    coefficient_clip=cfg.eggroll_coefficient_clip, max_delta_rms=cfg.eggroll_max_delta_rms)
            evals += cfg.eggroll_population_size
        steps += 1
    el = (time.perf_counter() - t0) * 1e3
    xl, yl = batches(cfg.max_iters - 1)
    r.update(final_train_loss=_loss(m, xl, yl), final_loss=_loss(m, *held), elapsed_ms=el, train_steps=steps,
             forward_evaluations=evals)
    r["loss_delta"] = r["initial_loss"] - r["final_loss"]
    r["train_loss_delta"] = r["initial_train_loss"] - r["final_train_loss"]
    r["evaluations_per_second"] = evals / (el / 1e3) if el > 0 else float("inf")
    r["milliseconds_per_train_step"] = el / steps if steps else float("inf")
    r["loss_delta_per_forward_evaluation"] = r["loss_delta"] / evals if evals else 0.0
    r["loss_delta_per_second"] = r["loss_delta"] / (el / 1e3) if el > 0 else 0.0
    return r


def run_optimizer_dynamics_pair(make_model, batches, held, cfg: OptimizerDynamicsConfig) -> dict:
    return {"config": asdict(cfg), "adamw": run_optimizer_dynamics("adamw", make_model, batches, held, cfg),
            "eggroll": run_optimizer_dynamics("eggroll", make_model, batches, held, cfg)}

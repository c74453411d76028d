"""Recurrent-state predictive coding (``training.predictive_coding``): inference of the
state entering a chunk, amortised into the ordinary recurrence.

Reference: burn_dragon_language/src/train/steps.rs:775-1000 (cadence, amortisation
constraint, state update), :3593-3960 (oracle and observed-prefix corrections) and the
TBPTT chunk loop :11990-12120; config schema.rs PredictiveCodingConfig.

Per due chunk, with the ``observed_prefix`` contract (causal; the default):

1. the chunk runs forward from the incoming state rho_in as usual (student exit state);
2. a detached copy of rho_in takes ``steps`` SGD steps on the chunk's own next-token
   CE over its observed tokens (inputs[:-1] -> inputs[1:]); the update rule is the PC
   inference rule (gradient + ``latent_decay`` * rho, norm clip at ``max_grad_norm``
   per sample or over the whole tensor, times ``step_size``);
3. the chunk is replayed from the corrected rho_in (no gradient): the teacher exit state;
4. ``parameter_update = "optimizer"``: the amortisation constraint
   ``relu(mean (s - t)^2 / (mean s^2 + mean t^2) - tolerance^2)`` (scale not
   differentiated), averaged over layers, on up to
   ``amortization_max_state_slots`` latent slots of every layer's rho (a rotating
   subset) joins the chunk loss, so the learned transition moves toward the inferred
   state; ``"state_only_control"``: the teacher exit state replaces the student's and
   the weights are not asked to amortise it.

The ``oracle_next_token_negative_control`` contract corrects rho_in with the chunk's
targets before the forward (non-causal; it needs ``allow_oracle_target_leak``).
Chunks are due every ``apply_every_chunks`` (observed prefix: when ordinal + 1 is a
multiple; oracle: when the ordinal is), from ``warmup_steps`` on.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models import reference as R
from ..models.state import ModelState


@dataclass
class RecurrentStatePCConfig:
    enabled: bool = False
    mode: str = "recurrent_state"
    state_scope: str = "core"  # core | all (rho is the only state on the BDH path)
    backward_mode: str = "chunked"  # chunked | block (one chunk per step here: the same)
    parameter_update: str = "optimizer"  # optimizer | state_only_control (alias: frozen)
    observation_contract: str = "observed_prefix"  # | oracle_next_token_negative_control
    allow_oracle_target_leak: bool = False
    steps: int = 1
    step_size: float = 0.1
    latent_decay: float = 0.0
    max_grad_norm: float | None = 1.0
    gradient_norm_scope: str = "per_sample"  # per_sample | global
    eps: float = 1e-8
    apply_every_chunks: int = 1
    amortization_tolerance: float = 0.05
    amortization_max_state_slots: int = 64
    warmup_steps: int = 0
    sync_diagnostics: bool = False

    def validate(self) -> None:
        if self.parameter_update == "frozen":
            self.parameter_update = "state_only_control"
        if self.mode != "recurrent_state":
            raise ValueError(f"training.predictive_coding.mode {self.mode!r}")
        if self.parameter_update not in ("optimizer", "state_only_control"):
            raise ValueError(f"training.predictive_coding.parameter_update {self.parameter_update!r}")
        if self.observation_contract not in ("observed_prefix", "oracle_next_token_negative_control"):
            raise ValueError(f"training.predictive_coding.observation_contract {self.observation_contract!r}")
        if self.observation_contract == "oracle_next_token_negative_control" and not self.allow_oracle_target_leak:
            raise ValueError("the oracle contract reads the chunk's targets: set "
                             "training.predictive_coding.allow_oracle_target_leak = true to run it")
        if self.steps <= 0 or self.apply_every_chunks <= 0:
            raise ValueError("training.predictive_coding.steps and apply_every_chunks must be > 0")


def chunk_due(cfg: RecurrentStatePCConfig, ordinal: int) -> bool:
    if not cfg.enabled or ordinal < cfg.warmup_steps:
        return False
    c = max(cfg.apply_every_chunks, 1)
    return (ordinal + 1) % c == 0 if cfg.observation_contract == "observed_prefix" else ordinal % c == 0


def pc_sgd(r: torch.Tensor, g: torch.Tensor, cfg: RecurrentStatePCConfig) -> torch.Tensor:
    if cfg.latent_decay:
        g = g + cfg.latent_decay * r
    if cfg.max_grad_norm is not None:
        if cfg.gradient_norm_scope == "per_sample":
            n = g.reshape(g.shape[0], -1).norm(dim=1).view(-1, *([1] * (g.dim() - 1)))
        else:
            n = g.norm()
        g = g * (cfg.max_grad_norm / (n + cfg.eps)).clamp(max=1.0)
    return r - cfg.step_size * g


def _ce(model, x, y, rhos):
    st = ModelState(list(rhos), 0)
    return R.cross_entropy(model(x, state=st), y), st


def correct_entry(model, rhos, x, y, cfg: RecurrentStatePCConfig) -> list[torch.Tensor]:
    """``steps`` PC inference steps on the entry state (weights held fixed)."""
    cur = [r.detach() for r in rhos]
    for _ in range(cfg.steps):
        leaves = [r.clone().requires_grad_(True) for r in cur]
        energy, _ = _ce(model, x, y, leaves)
        grads = torch.autograd.grad(energy, leaves, allow_unused=True)
        cur = [r.detach() if g is None else pc_sgd(r.detach(), g, cfg).detach() for r, g in zip(leaves, grads)]
    return cur


def amortization_constraint(student, teacher, cfg: RecurrentStatePCConfig, step: int):
    total, n = None, 0
    for s, t in zip(student, teacher):
        if s is None or t is None or s.shape != t.shape:
            continue
        t = t.detach()
        slots = s.shape[2]
        k = min(max(cfg.amortization_max_state_slots, 1), slots)
        stride = max(slots // k, 1)
        idx = torch.tensor(sorted({(step + i * stride) % slots for i in range(k)}), device=s.device)
        ss, tt = s.index_select(2, idx), t.index_select(2, idx)
        scale = (ss.detach().pow(2).mean() + tt.pow(2).mean()).clamp_min(max(cfg.eps, 1e-12))
        v = ((ss - tt).pow(2).mean() / scale - max(cfg.amortization_tolerance, 0.0) ** 2).clamp_min(0.0)
        total = v if total is None else total + v
        n += 1
    return None if total is None else total / n


def state_pc_chunk_loss(model, x, y, state: ModelState, cfg: RecurrentStatePCConfig, ordinal: int):
    """The chunk's training loss (with the parameter graph) and the state it hands on;
    ``state`` is the incoming state (detached). Returns (loss, next_state, report)."""
    rep = {"corrected": False}
    due = chunk_due(cfg, ordinal) and state.rhos is not None
    if due and cfg.observation_contract == "oracle_next_token_negative_control":
        state = ModelState(correct_entry(model, state.rhos, x, y, cfg), state.position)
        rep["corrected"] = True
    entry = None if state.rhos is None else [r.detach() for r in state.rhos]
    loss = model.loss(x, y, state=state)  # advances state.rhos (student exit, with graph)
    if due and cfg.observation_contract == "observed_prefix" and x.shape[1] >= 2:
        fixed = correct_entry(model, entry, x[:, :-1], x[:, 1:], cfg)
        with torch.no_grad():
            replay = ModelState(list(fixed), 0)
            model(x, state=replay)
        rep["corrected"] = True
        if cfg.parameter_update == "optimizer":
            c = amortization_constraint(state.rhos, replay.rhos, cfg, ordinal)
            if c is not None:
                rep["amortization_loss"] = float(c.detach())
                loss = loss + c
        else:
            state.rhos = [r.detach() for r in replay.rhos]
    return loss, state, rep

"""Stream-warm validation with a recurrent-state carry probe.

Reference: the event scheduler's stream validation (burn_dragon_language/src/train/
schedule.rs:3180-3320; config ``training.sequence_state_probe`` {enabled,
paired_batches, max_rho_slots}, schema.rs SequenceStateProbeConfig). Validation walks
consecutive chunks of held-out streams with the recurrent state carried from chunk to
chunk (reset where a new document starts): the mean of those losses is the warm loss.
For the first ``paired_batches`` chunks that continue a stream, the same chunk is also
scored from a fresh state (cold). ``carry_nll_gain`` = cold - warm on those pairs and
``carry_relative_gain`` = gain / |cold| say how much the carried state helps. A state
summary (per layer rms / |max| / fraction non-zero of rho, at most ``max_rho_slots``
layers) is attached.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.state import ModelState
from ..utils.diagnostics import state_summary


@dataclass
class SequenceStateProbeConfig:
    enabled: bool = False
    paired_batches: int = 4
    max_rho_slots: int = 8


@torch.no_grad()
def stream_warm_validation(model, stream, chunks: int, probe: SequenceStateProbeConfig, device) -> dict:
    """``model``: a ``BDH`` (``model.loss(x, y, state=...)``); ``stream``: an object whose
    ``next()`` returns (inputs, targets, reset) chunks of consecutive stream positions."""
    state = ModelState.empty()
    total, count = 0.0, 0
    warm_p, cold_p, paired = 0.0, 0.0, 0
    for _ in range(chunks):
        x, y, reset = stream.next()
        x, y = x.to(device), y.to(device)
        if reset:
            state = ModelState.empty()
        pair = probe.enabled and not reset and paired < probe.paired_batches
        loss = float(model.loss(x, y, state=state))
        total, count = total + loss, count + 1
        if pair:
            cold = float(model.loss(x, y, state=ModelState.empty()))
            warm_p, cold_p, paired = warm_p + loss, cold_p + cold, paired + 1
    out = {"warm_loss": total / count if count else None, "paired_batches": paired}
    if paired:
        w, c = warm_p / paired, cold_p / paired
        gain = c - w
        out.update(paired_warm_loss=w, paired_cold_loss=c, carry_nll_gain=gain,
                   carry_relative_gain=0.0 if abs(c) <= 2.220446049250313e-16 else gain / abs(c))
    if probe.enabled and state.rhos is not None:
        out["state"] = [{"layer_index": i, **state_summary(r)} for i, r in
                        enumerate(state.rhos[:max(probe.max_rho_slots, 0)])]
    return out

"""Startup batch-size selection.

The reference probes candidate batch sizes by running training steps and reading the
device's memory high-water mark, predicting larger candidates from smaller probes
(burn_dragon_language/src/train/startup_autotune.rs). Here the fused step's device
memory is fully determined by its workspace, which is allocated up front with known
shapes, so the footprint of a candidate batch is computed exactly: the workspace is
built on the ``meta`` device (no memory touched) and its tensors are summed, plus the
parameter store (fp32 weights, fp32 grads, bf16 shadow) and the two AdamW moments.
Selection is then a binary search over batch sizes against the budget

    budget = target_device_memory_mb (if set) else free device memory / safety margin

capped by ``max_batch_size``; an optional measured probe (``probe_steps`` > 0 on a GPU)
runs real steps at the chosen size and backs off by halving if the measured high-water
mark exceeds the budget. ``target_effective_batch_size`` then sets gradient
accumulation = ceil(target / batch).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..config import AutoBatchSizeConfig, DragonConfig


def _tensor_bytes(obj, seen: set) -> int:
    total = 0
    items = obj if isinstance(obj, (list, tuple)) else [obj]
    for t in items:
        if isinstance(t, torch.Tensor) and id(t) not in seen:
            seen.add(id(t))
            total += t.numel() * t.element_size()
        elif isinstance(t, (list, tuple)):
            total += _tensor_bytes(t, seen)
    return total


def workspace_bytes(cfg: DragonConfig, batch: int, block: int) -> int:
    """Device bytes of the fused step's activation workspace for [batch, block]."""
    from ..models.bdh_fused import FusedWorkspace

    ws = FusedWorkspace(cfg, batch, block, torch.device("meta"))
    seen: set = set()
    return sum(_tensor_bytes(v, seen) for v in vars(ws).values())


def state_bytes(cfg: DragonConfig) -> int:
    """Parameters (fp32 data + fp32 grad + bf16 shadow) and AdamW m, v."""
    from ..models.bdh import param_shapes

    n = sum(math.prod(s) for s in param_shapes(cfg).values())
    return n * (4 + 4 + 2 + 4 + 4)


@dataclass
class AutoBatchResult:
    batch_size: int
    gradient_accumulation_steps: int
    predicted_bytes: int
    budget_bytes: int
    measured_bytes: int | None = None


def choose_batch_size(cfg: DragonConfig, block: int, ab: AutoBatchSizeConfig, budget_bytes: int | None = None,
                      target_effective_batch: int | None = None, granularity: int = 1) -> AutoBatchResult:
    """Largest batch (a multiple of ``granularity``) whose predicted footprint times the
    safety margin fits the budget."""
    if budget_bytes is None:
        if ab.target_device_memory_mb:
            budget_bytes = ab.target_device_memory_mb * 2 ** 20
        elif torch.cuda.is_available():
            free, _ = torch.cuda.mem_get_info()
            budget_bytes = int(free / max(ab.probe_safety_margin, 1.0))
        else:
            raise ValueError("auto_batch_size needs target_device_memory_mb without a GPU")
    fixed = state_bytes(cfg)

    def fits(b: int) -> bool:
        return (fixed + workspace_bytes(cfg, b, block)) * max(ab.probe_safety_margin, 1.0) <= budget_bytes

    lo = max(ab.min_batch_size, granularity)
    hi = ab.max_batch_size or 4096
    hi -= hi % granularity
    if not fits(lo):
        raise ValueError(f"auto_batch_size: even batch {lo} needs "
                         f"{(fixed + workspace_bytes(cfg, lo, block)) / 2**20:.0f} MiB > budget "
                         f"{budget_bytes / 2**20:.0f} MiB")
    best = lo
    if ab.binary_search:
        a, b = lo // granularity, hi // granularity
        while a <= b:
            mid = (a + b) // 2
            if fits(mid * granularity):
                best, a = mid * granularity, mid + 1
            else:
                b = mid - 1
    else:
        c = lo
        while c <= hi and fits(c):
            best, c = c, c + granularity
    acc = 1
    if target_effective_batch:
        acc = max(1, -(-target_effective_batch // best))
    return AutoBatchResult(best, acc, fixed + workspace_bytes(cfg, best, block), budget_bytes)


def probe(trainer, batch: int, block: int, steps: int, vocab: int) -> int:
    """Run ``steps`` real steps at ``batch`` and return the device high-water mark."""
    dev = trainer.device
    torch.cuda.reset_peak_memory_stats(dev)
    x = torch.randint(0, vocab, (batch, block), device=dev)
    for _ in range(max(steps, 1)):
        trainer.compute_grads(x, x)
    torch.cuda.synchronize(dev)
    return torch.cuda.max_memory_allocated(dev)

"""Controlled continual-learning benchmark on context-identifiable recurrences.

Reference: burn_dragon_language/src/train/continual_benchmark.rs:1-440. Four tasks A-D
each generate payload streams by a second-order recurrence mod ``payload_modulus``:
x_n = (a x_{n-1} + b x_{n-2} + c) mod m with (a, b, c) = (1,1,1), (3,1,2), (1,3,3),
(3,3,1); tokens are payload + 1. Every row starts with two seeded values, and the first
``observation_tokens(T)`` tokens (half the block, clamped to [3, 16]) are an observed
support prefix: the loss mask starts at the last of them, so the active recurrence is
identifiable before supervised tokens begin. Seeding follows the reference
(SplitMix64 of a row key mixing the split seed, batch index and row) so the same spec
yields the same batches.

Also: the task-ID-free stream descriptor (counts of observed transitions consistent
with each small (a, b, c), minus chance, unit-normalised), a streaming context selector
over those descriptors (cosine novelty threshold, EMA centroids) and balanced sparse
context masks; ``run_sequential`` trains tasks in order and reports each task's
held-out masked loss / accuracy after every phase (the forgetting matrix).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

_M64 = (1 << 64) - 1
PAYLOAD_OFFSET = 1
DESCRIPTOR_LIMIT = 8
MAX_OBSERVATION = 16
TASKS = {"a": (1, 1, 1), "b": (3, 1, 2), "c": (1, 3, 3), "d": (3, 3, 1)}


def splitmix64(x: int) -> int:
    """SplitMix64 (Steele, Lea and Flood 2014; the finaliser used by Vigna's xorshift+)."""
    x = (x + 0x9E3779B97F4A7C15) & _M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _M64
    return x ^ (x >> 31)


def observation_tokens(block: int) -> int:
    half = -(-block // 2)
    return 3 if half < 3 else min(half, MAX_OBSERVATION)


@dataclass
class ContextRecurrenceSpec:
    batch_size: int = 32
    block_size: int = 32
    payload_modulus: int = 16

    def validate(self) -> None:
        if self.batch_size <= 0 or self.block_size < 4 or self.payload_modulus < 4:
            raise ValueError("context recurrence needs batch_size > 0, block_size >= 4, payload_modulus >= 4")

    @property
    def vocab_size(self) -> int:
        return PAYLOAD_OFFSET + self.payload_modulus


def _sequence(task: str, split_seed: int, batch_index: int, row: int, block: int, m: int) -> list[int]:
    key = split_seed ^ ((batch_index * 0xD6E8FEB86659FD93) & _M64) ^ ((row * 0xA0761D6478BD642F) & _M64)
    vals = [splitmix64(key) % m, splitmix64(key ^ 0x589965CC75374CC3) % m]
    a, b, c = TASKS[task]
    while len(vals) <= block:
        vals.append((a * vals[-1] + b * vals[-2] + c) % m)
    return [v + PAYLOAD_OFFSET for v in vals]


def batch(task: str, spec: ContextRecurrenceSpec, split_seed: int, batch_index: int):
    """(inputs [B, T], targets [B, T], loss_mask [B, T], descriptor) of one task."""
    spec.validate()
    rows = [_sequence(task, split_seed, batch_index, r, spec.block_size, spec.payload_modulus)
            for r in range(spec.batch_size)]
    t = torch.tensor(rows, dtype=torch.long)
    start = observation_tokens(spec.block_size) - 1
    mask = (torch.arange(spec.block_size) >= start).long().expand(spec.batch_size, -1).contiguous()
    x = t[:, :spec.block_size].contiguous()
    return x, t[:, 1:].contiguous(), mask, stream_descriptor(x, spec)


def _normalize(v: torch.Tensor) -> torch.Tensor:
    n = v.norm()
    return v / n if float(n) > 0 else v


def stream_descriptor(inputs: torch.Tensor, spec: ContextRecurrenceSpec) -> torch.Tensor:
    m = spec.payload_modulus
    span = min(m, DESCRIPTOR_LIMIT)
    obs = observation_tokens(spec.block_size)
    d = torch.full((span ** 3,), -(inputs.shape[0] * (obs - 2)) / m, dtype=torch.float64)
    p = (inputs[:, :obs] - PAYLOAD_OFFSET).tolist()
    for row in p:
        for pp, prev, nxt in zip(row, row[1:], row[2:]):
            for a in range(span):
                for b in range(span):
                    c = (nxt + m - (a * prev + b * pp) % m) % m
                    if c < span:
                        d[(a * span + b) * span + c] += 1.0
    return _normalize(d).float()


class StreamingContextSelector:
    """Nearest-centroid context memory with novelty creation (cosine below the threshold
    makes a new context; the chosen centroid follows the descriptor at ``update_rate``)."""

    def __init__(self, novelty_cosine_threshold: float = 0.8, centroid_update_rate: float = 0.1):
        if not -1.0 <= novelty_cosine_threshold <= 1.0 or not 0.0 <= centroid_update_rate <= 1.0:
            raise ValueError("streaming context selector thresholds out of range")
        self.thr, self.rate = novelty_cosine_threshold, centroid_update_rate
        self.centroids: list[torch.Tensor] = []

    def select(self, desc: torch.Tensor, allow_create: bool = True) -> dict:
        if abs(float(desc.norm()) - 1.0) > 1e-3:
            raise ValueError("streaming context descriptor must be unit normalised")
        sims = [float(c @ desc) for c in self.centroids]
        best = max(range(len(sims)), key=sims.__getitem__) if sims else None
        if (best is None or sims[best] < self.thr) and allow_create:
            self.centroids.append(_normalize(desc.clone()))
            return {"context_index": len(self.centroids) - 1, "created": True,
                    "cosine_similarity": 0.0 if best is None else sims[best]}
        if best is None:
            raise ValueError("no context yet and creation is disabled")
        if allow_create and self.rate > 0:
            self.centroids[best] = _normalize(self.centroids[best] * (1 - self.rate) + desc * self.rate)
        return {"context_index": best, "created": False, "cosine_similarity": sims[best]}


def balanced_context_mask(seed: int, index: int, width: int, active_fraction: float,
                          prior: list[torch.Tensor]) -> torch.Tensor:
    """``active_fraction`` of ``width`` channels, least-used first (ties by a seeded hash):
    contexts stay disjoint while free capacity remains, then reuse is balanced."""
    if width <= 0 or not 0.0 < active_fraction <= 1.0 or index != len(prior):
        raise ValueError("balanced context masks: width > 0, fraction in (0, 1], sequential indices")
    k = min(max(round(width * active_fraction), 1), width)
    usage = [0] * width
    for mk in prior:
        for i, v in enumerate(mk.tolist()):
            usage[i] += v > 0
    key = lambda i: (usage[i], splitmix64(seed ^ ((index * 0xD6E8FEB86659FD93) & _M64)  # noqa: E731
                                          ^ ((i * 0xA0761D6478BD642F) & _M64)), i)
    out = torch.zeros(width)
    out[sorted(range(width), key=key)[:k]] = 1.0
    return out


@torch.no_grad()
def evaluate(model, task: str, spec: ContextRecurrenceSpec, seed: int, batches: int = 2) -> dict:
    loss = acc = n = 0.0
    for i in range(batches):
        x, y, mask, _ = batch(task, spec, seed, i)
        lg = model(x)
        lp = torch.log_softmax(lg.float(), -1)
        nll = -lp.gather(-1, y.unsqueeze(-1)).squeeze(-1)
        mk = mask.float()
        loss += float((nll * mk).sum())
        acc += float(((lg.argmax(-1) == y).float() * mk).sum())
        n += float(mk.sum())
    return {"loss": loss / n, "accuracy": acc / n}


def run_sequential(trainer, spec: ContextRecurrenceSpec, tasks=("a", "b", "c", "d"), steps_per_task: int = 50,
                   train_seed: int = 1, holdout_seed: int = 2) -> dict:
    """Train ``trainer`` (``trainer.step(x, y, mask)``) on each task in turn; after every
    phase evaluate all tasks on held-out batches. Returns the matrix and forgetting
    (final minus best accuracy per task)."""
    matrix = []
    for ti, task in enumerate(tasks):
        for s in range(steps_per_task):
            x, y, mask, _ = batch(task, spec, train_seed + 7919 * ti, s)
            trainer.step(x, y, mask)
        matrix.append({t: evaluate(trainer.model, t, spec, holdout_seed) for t in tasks})
    forgetting = {t: matrix[-1][t]["accuracy"] - max(row[t]["accuracy"] for row in matrix) for t in tasks}
    return {"after_phase": matrix, "forgetting": forgetting}


def acquisition(before: dict, after: dict) -> dict:
    """A task's acquisition over a phase: loss reduction and accuracy gain."""
    return {"loss_reduction": before["loss"] - after["loss"], "accuracy_gain": after["accuracy"] - before["accuracy"]}


def acquisition_gate(baseline: list[dict], candidate: list[dict], loss_floor_ratio: float = 0.9,
                     accuracy_tolerance: float = 0.0, minimum_baseline_loss_reduction: float = 0.0,
                     minimum_baseline_accuracy_gain: float = 0.0) -> dict:
    """Does a candidate method acquire every task as well as the baseline did
    (continual_benchmark.rs:439-520)? A task counts only if the baseline acquired it
    (loss reduction and accuracy gain at least the minimums); the candidate must keep at
    least ``loss_floor_ratio`` of the baseline's loss reduction and its accuracy gain
    within ``accuracy_tolerance``."""
    if not baseline or len(baseline) != len(candidate):
        raise ValueError("continual acquisition vectors must be non-empty and equally sized")
    if not 0.0 <= loss_floor_ratio <= 1.0 or min(accuracy_tolerance, minimum_baseline_loss_reduction,
                                                  minimum_baseline_accuracy_gain) < 0:
        raise ValueError("continual acquisition thresholds must be non-negative, loss_floor_ratio in [0, 1]")
    matched, acquired, ratios, deltas = True, [], [], []
    for b, c in zip(baseline, candidate):
        ok = b["loss_reduction"] >= minimum_baseline_loss_reduction and \
            b["accuracy_gain"] >= minimum_baseline_accuracy_gain
        ratios.append(c["loss_reduction"] / b["loss_reduction"] if abs(b["loss_reduction"]) > 1e-12 else 0.0)
        deltas.append(c["accuracy_gain"] - b["accuracy_gain"])
        matched &= ok and c["loss_reduction"] >= b["loss_reduction"] * loss_floor_ratio \
            and c["accuracy_gain"] + accuracy_tolerance >= b["accuracy_gain"]
        acquired.append(ok)
    return {"matched": matched, "baseline_acquired": acquired, "loss_ratios": ratios, "accuracy_deltas": deltas}

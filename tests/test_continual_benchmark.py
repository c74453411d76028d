"""Continual-learning benchmark (CPU): recurrences, masks, descriptors, the context
selector, balanced masks and a short sequential run."""

import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.train.continual_benchmark import (ContextRecurrenceSpec, StreamingContextSelector,
                                                        balanced_context_mask, batch, observation_tokens,
                                                        run_sequential, splitmix64)
from burn_dragon_b200.train.trainer import Trainer


def test_splitmix64_known_values():
    # the first outputs of SplitMix64 seeded with 0 (state advanced once per call)
    assert splitmix64(0) == 0xE220A8397B1DCDAF
    assert splitmix64(0x9E3779B97F4A7C15) == 0x6E789E6AA1B965F4


def test_batches_follow_the_recurrence_and_mask_the_prefix():
    spec = ContextRecurrenceSpec(batch_size=3, block_size=10, payload_modulus=16)
    assert observation_tokens(10) == 5 and observation_tokens(4) == 3 and observation_tokens(64) == 16
    x, y, mask, d = batch("b", spec, 11, 0)
    full = torch.cat([x, y[:, -1:]], 1) - 1
    for r in full.tolist():
        for i in range(2, len(r)):
            assert r[i] == (3 * r[i - 1] + 1 * r[i - 2] + 2) % 16
    assert mask[0].tolist() == [0] * 4 + [1] * 6
    assert torch.equal(batch("b", spec, 11, 0)[0], x) and not torch.equal(batch("b", spec, 12, 0)[0], x)
    assert abs(float(d.norm()) - 1.0) < 1e-5


def test_selector_separates_tasks_and_masks_balance():
    spec = ContextRecurrenceSpec(batch_size=8, block_size=32, payload_modulus=16)
    # same-task batches of this size score ~0.7-0.8, different tasks ~0.35 or less
    sel = StreamingContextSelector(novelty_cosine_threshold=0.5)
    ids = [sel.select(batch(t, spec, 5, i)[3])["context_index"] for t in "abcd" for i in range(2)]
    assert ids == [0, 0, 1, 1, 2, 2, 3, 3]
    m0 = balanced_context_mask(3, 0, 8, 0.5, [])
    m1 = balanced_context_mask(3, 1, 8, 0.5, [m0])
    assert m0.sum() == 4 and float((m0 * m1).sum()) == 0.0  # disjoint while capacity remains


def test_sequential_run_reports_a_forgetting_matrix():
    spec = ContextRecurrenceSpec(batch_size=4, block_size=16, payload_modulus=8)
    cfg = DragonConfig(n_layer=1, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, vocab_size=spec.vocab_size,
                       dropout=0.0)
    rep = run_sequential(Trainer(cfg, "cpu", lr=1e-2, seed=0), spec, tasks=("a", "b"), steps_per_task=3)
    assert len(rep["after_phase"]) == 2 and set(rep["forgetting"]) == {"a", "b"}
    assert all(v <= 0 for v in rep["forgetting"].values())


def test_acquisition_gate():
    from burn_dragon_b200.train.continual_benchmark import acquisition, acquisition_gate

    base = [acquisition({"loss": 2.0, "accuracy": 0.1}, {"loss": 1.0, "accuracy": 0.6}),
            {"loss_reduction": 0.5, "accuracy_gain": 0.2}]
    good = [{"loss_reduction": 0.95, "accuracy_gain": 0.5}, {"loss_reduction": 0.5, "accuracy_gain": 0.2}]
    bad = [{"loss_reduction": 0.5, "accuracy_gain": 0.5}, {"loss_reduction": 0.5, "accuracy_gain": 0.2}]
    g = acquisition_gate(base, good, loss_floor_ratio=0.9)
    assert g["matched"] and abs(g["loss_ratios"][0] - 0.95) < 1e-12
    assert not acquisition_gate(base, bad, loss_floor_ratio=0.9)["matched"]
    assert not acquisition_gate(base, good, minimum_baseline_accuracy_gain=0.3)["matched"]


def test_benchmark_clis():
    from burn_dragon_b200.cli.continual_benchmark import main as cb
    from burn_dragon_b200.cli.optimizer_dynamics import main as od

    out = cb(["--tasks", "ab", "--steps-per-task", "2", "--batch-size", "4", "--block-size", "16", "--n-layer", "1",
              "--n-embd", "16", "--n-head", "2", "--latent-total", "64"])
    assert len(out["after_phase"]) == 2 and set(out["forgetting"]) == {"a", "b"}
    out = od(["--max-iters", "2", "--population", "4", "--rank", "2", "--n-embd", "16"])
    assert out["adamw"]["train_steps"] == out["eggroll"]["train_steps"] == 2

"""AdamW vs EGGROLL dynamics report and the EGGROLL update options (CPU)."""

import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.train.eggroll import normalize_fitness
from burn_dragon_b200.train.optimizer_dynamics import OptimizerDynamicsConfig, run_optimizer_dynamics_pair


def test_fitness_normalizations():
    f = torch.tensor([3.0, -1.0, 2.0, 10.0])
    torch.testing.assert_close(normalize_fitness(f, "center"), f - 3.5)
    # ranks 2, 0, 1, 3 of 4 -> r / 3 - 0.5
    torch.testing.assert_close(normalize_fitness(f, "rank"), torch.tensor([2.0, 0.0, 1.0, 3.0]) / 3 - 0.5)


def test_dynamics_pair_report():
    cfg = DragonConfig(n_layer=1, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, vocab_size=16, dropout=0.0)
    g = torch.Generator().manual_seed(0)
    # a learnable stream: each token is the previous plus one
    base = torch.randint(0, 16, (8, 1), generator=g)
    seq = (base + torch.arange(17)) % 16
    batches = lambda i: (seq[:, :-1], seq[:, 1:])  # noqa: E731
    d = OptimizerDynamicsConfig(max_iters=6, eggroll_population_size=8, eggroll_rank=2)
    rep = run_optimizer_dynamics_pair(lambda: BDH(cfg, seed=1), batches, (seq[:, :-1], seq[:, 1:]), d)
    a, e = rep["adamw"], rep["eggroll"]
    assert a["forward_evaluations"] == 6 and e["forward_evaluations"] == 48
    assert a["loss_delta"] > 0  # AdamW learns the pattern within a few steps
    for r in (a, e):
        assert abs(r["loss_delta"] - (r["initial_loss"] - r["final_loss"])) < 1e-9 and r["train_steps"] == 6


def test_deepcopy_keeps_parameters_on_the_copied_store():
    import copy

    from burn_dragon_b200.train.optim import FusedAdamW

    cfg = DragonConfig(n_layer=1, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, vocab_size=16, dropout=0.0)
    m = BDH(cfg, seed=1)
    with torch.no_grad():
        m.encoder.add_(0.5)
    t = copy.deepcopy(m)
    torch.testing.assert_close(t.encoder, m.encoder)
    t.store.grad.fill_(1.0)
    FusedAdamW(t.store, lr=0.1).step()
    assert not torch.equal(t.encoder, m.encoder)  # the copy's optimizer moves the copy's parameters
    torch.testing.assert_close(m.store.view(m.store.data, "encoder"), m.encoder)

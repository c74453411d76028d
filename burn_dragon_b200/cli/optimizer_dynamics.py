"""AdamW vs EGGROLL dynamics CLI: the same small BDH and synthetic recurrence data
trained with both optimizers; prints both reports as JSON
(burn_dragon_language/src/train/optimizer_dynamics.rs).

  python -m burn_dragon_b200.cli.optimizer_dynamics [--max-iters 64] [--population 64] [--rank 4]
         [--sigma 0.01] [--adamw-lr 0.025] [--eggroll-lr 0.1] [--fitness rank|center|none] [--seed 29]
"""

from __future__ import annotations

import argparse
import json

from ..config import DragonConfig
from ..models.bdh import BDH
from ..train.continual_benchmark import ContextRecurrenceSpec, batch
from ..train.optimizer_dynamics import OptimizerDynamicsConfig, run_optimizer_dynamics_pair


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--max-iters", type=int, default=64)
    ap.add_argument("--population", type=int, default=64)
    ap.add_argument("--rank", type=int, default=4)
    ap.add_argument("--sigma", type=float, default=1e-2)
    ap.add_argument("--adamw-lr", type=float, default=2.5e-2)
    ap.add_argument("--eggroll-lr", type=float, default=1e-1)
    ap.add_argument("--fitness", choices=("rank", "center", "none"), default="rank")
    ap.add_argument("--seed", type=int, default=29)
    ap.add_argument("--n-embd", type=int, default=32)
    a = ap.parse_args(argv)
    spec = ContextRecurrenceSpec(batch_size=8, block_size=16, payload_modulus=8)
    cfg = DragonConfig(n_layer=1, n_embd=a.n_embd, n_head=2, mlp_internal_dim_multiplier=4,
                       vocab_size=spec.vocab_size, dropout=0.0)
    d = OptimizerDynamicsConfig(max_iters=a.max_iters, seed=a.seed, adamw_learning_rate=a.adamw_lr,
                                eggroll_learning_rate=a.eggroll_lr, eggroll_sigma=a.sigma,
                                eggroll_population_size=a.population, eggroll_rank=a.rank,
                                eggroll_fitness_normalization=a.fitness)

    def batches(i):
        x, y, _, _ = batch("a", spec, a.seed, i)
        return x, y

    held = batch("a", spec, a.seed + 1, 0)[:2]
    out = run_optimizer_dynamics_pair(lambda: BDH(cfg, seed=a.seed), batches, held, d)
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()

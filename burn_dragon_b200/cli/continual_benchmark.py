"""Continual-learning benchmark CLI: trains a small BDH on the recurrence tasks in order
and prints the per-phase held-out loss / accuracy matrix and the forgetting per task as
one JSON document (the reference's controlled continual benchmark,
burn_dragon_language/src/train/continual_benchmark.rs).

  python -m burn_dragon_b200.cli.continual_benchmark [--tasks abcd] [--steps-per-task 100]
         [--batch-size 32 --block-size 32 --payload-modulus 16]
         [--n-layer 2 --n-embd 64 --n-head 4 --latent-total 1024] [--lr 3e-3] [--seed 1] [--backend cpu|cuda]
"""

from __future__ import annotations

import argparse
import json

import torch

from ..config import DragonConfig
from ..train.continual_benchmark import ContextRecurrenceSpec, run_sequential
from ..train.trainer import Trainer


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tasks", default="abcd")
    ap.add_argument("--steps-per-task", type=int, default=100)
    ap.add_argument("--batch-size", type=int, default=32)
    ap.add_argument("--block-size", type=int, default=32)
    ap.add_argument("--payload-modulus", type=int, default=16)
    ap.add_argument("--n-layer", type=int, default=2)
    ap.add_argument("--n-embd", type=int, default=64)
    ap.add_argument("--n-head", type=int, default=4)
    ap.add_argument("--latent-total", type=int, default=1024)
    ap.add_argument("--lr", type=float, default=3e-3)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--backend", choices=("cpu", "cuda"), default="cpu")
    a = ap.parse_args(argv)
    spec = ContextRecurrenceSpec(a.batch_size, a.block_size, a.payload_modulus)
    cfg = DragonConfig(n_layer=a.n_layer, n_embd=a.n_embd, n_head=a.n_head,
                       mlp_internal_dim_multiplier=a.latent_total // a.n_embd, vocab_size=spec.vocab_size, dropout=0.0)
    cfg.validate()
    dev = torch.device("cuda" if a.backend == "cuda" else "cpu")
    tr = Trainer(cfg, dev, lr=a.lr, seed=a.seed)
    rep = run_sequential(tr, spec, tasks=tuple(a.tasks), steps_per_task=a.steps_per_task, train_seed=a.seed,
                         holdout_seed=a.seed + 1)
    out = {"spec": {"batch_size": spec.batch_size, "block_size": spec.block_size,
                    "payload_modulus": spec.payload_modulus}, "tasks": list(a.tasks), **rep}
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()

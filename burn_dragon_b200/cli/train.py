"""Training CLI (the reference's ``train_language`` example:
burn_dragon_language/examples/train_language.rs:1-226).

  python -m burn_dragon_b200.cli.train --config base.toml [--config overlay.toml]
         [--set training.max_iters=100 --set optimizer.learning_rate=3e-4] [--run-name NAME]
         [--backend cuda|cpu] [--seed S --n-layer L --n-embd D --n-head H --latent-total N
          --batch-size B --block-size T --max-iters K --checkpoint-interval-iters C]

Multi-GPU: launch with ``python -m torch.distributed.run --nproc-per-node N
--master-addr 127.0.0.1 -m burn_dragon_b200.cli.train ...``.
"""

from __future__ import annotations

import argparse
import json
import tomllib

from ..config import load_training_config


def parse_set(items: list[str]) -> dict:
    out: dict = {}
    for it in items:
        key, _, raw = it.partition("=")
        try:
            val = json.loads(raw)
        except json.JSONDecodeError:
            try:  # a TOML value: inline tables / arrays of tables, single-quoted strings
                val = tomllib.loads("v = " + raw)["v"]
            except tomllib.TOMLDecodeError:
                val = raw
        d = out
        parts = key.split(".")
        for p in parts[:-1]:
            d = d.setdefault(p, {})
        d[parts[-1]] = val
    return out


SHORTHANDS = (("--seed", "training.seed", int), ("--n-layer", "model.n_layer", int),
              ("--n-embd", "model.n_embd", int), ("--n-head", "model.n_head", int),
              ("--latent-total", "model.latent_total", int), ("--batch-size", "training.batch_size", int),
              ("--block-size", "training.block_size", int), ("--max-iters", "training.max_iters", int),
              ("--checkpoint-interval-iters", "training.checkpoint_interval_iters", int))


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", "--training-config", dest="config", action="append", required=True)
    ap.add_argument("--set", action="append", default=[])
    ap.add_argument("--run-name", default=None)
    ap.add_argument("--no-resume", action="store_true")
    ap.add_argument("--backend", choices=("cuda", "cpu"), default=None)
    # the reference's train_language shorthands (examples/train_language.rs:54-140)
    for flag, key, typ in SHORTHANDS:
        ap.add_argument(flag, dest=key.replace(".", "__"), type=typ, default=None)
    a = ap.parse_args(argv)
    overrides = parse_set(a.set)
    for flag, key, _ in SHORTHANDS:
        val = getattr(a, key.replace(".", "__"))
        if val is not None:
            sec, name = key.split(".")
            overrides.setdefault(sec, {})[name] = val
    cfg = load_training_config(a.config, overrides)
    from ..train.loop import train

    res = train(cfg, run_name=a.run_name, resume=not a.no_resume, backend=a.backend)
    print(json.dumps({k: v for k, v in res.items() if k != "profile"}))


if __name__ == "__main__":
    main()

"""Training CLI (the reference's ``train_language`` example:
burn_dragon_language/examples/train_language.rs:1-226).

  python -m burn_dragon_b200.cli.train --config base.toml [--config overlay.toml]
         [--set training.max_iters=100 --set optimizer.learning_rate=3e-4] [--run-name NAME]

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


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", action="append", required=True)
    ap.add_argument("--set", action="append", default=[])
    ap.add_argument("--run-name", default=None)
    ap.add_argument("--no-resume", action="store_true")
    a = ap.parse_args(argv)
    cfg = load_training_config(a.config, parse_set(a.set))
    from ..train.loop import train

    res = train(cfg, run_name=a.run_name, resume=not a.no_resume)
    print(json.dumps({k: v for k, v in res.items() if k != "profile"}))


if __name__ == "__main__":
    main()

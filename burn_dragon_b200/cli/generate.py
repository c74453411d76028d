"""Generation CLI: load a run's newest checkpoint and continue prompts, encoded and
decoded with the run's ``tokenizer.json`` (bytes or BPE).

  python -m burn_dragon_b200.cli.generate --run runs/cuda/NAME --prompt "hello" [--max-tokens 64]
         [--temperature 0.8 --top-k 40] [--batch 1]
"""

from __future__ import annotations

import argparse
import os

import torch

from ..config import training_config_from_dict
from ..models.bdh import BDH
from ..models.generate import Generator
from ..train.checkpoint import RunDir
from ..utils.tokenizer import load_tokenizer


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--run", required=True)
    ap.add_argument("--prompt", default="")
    ap.add_argument("--max-tokens", type=int, default=64)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--top-k", type=int, default=None)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    run = RunDir(a.run)
    cfg = training_config_from_dict(run.read_json("training_config.json"))
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    model = BDH(cfg.model, device=dev)
    if run.latest() is not None:
        run.load(None, model)
    tp = os.path.join(a.run, "tokenizer.json")
    tok = load_tokenizer(tp) if os.path.exists(tp) else load_tokenizer({"type": "byte"})
    prompt = tok.encode(a.prompt) or [0]
    x = torch.tensor([prompt] * a.batch, dtype=torch.long, device=dev)
    out = Generator(model).generate(x, a.max_tokens, temperature=a.temperature, top_k=a.top_k, seed=a.seed)
    for row in out.tolist():
        print(tok.decode(prompt + row))


if __name__ == "__main__":
    main()

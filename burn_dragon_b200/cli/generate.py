"""Generation CLI: load a run's newest checkpoint and continue prompts, encoded and
decoded with the run's ``tokenizer.json`` (bytes or BPE). Flags left unset take the
run's ``[generation]`` values (prompt, max_tokens, max_chars, temperature, top_k,
prompt_tokenizer / decode_tokenizer (the run's tokenizer, or one named in the config),
context_strategy, output_format: ``decoded_text`` prints text, ``token_ids`` prints the ids as JSON, ``auto``
is decoded text); burn_dragon_language/src/config/core.rs:18-60.

  python -m burn_dragon_b200.cli.generate --run runs/language/cuda/NAME --prompt "hello" [--max-tokens 64]
         [--temperature 0.8 --top-k 40] [--batch 1] [--output-format token_ids]
"""

from __future__ import annotations

import argparse
import json
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
    ap.add_argument("--prompt", default=None)
    ap.add_argument("--max-tokens", type=int, default=None)
    ap.add_argument("--max-chars", type=int, default=None)
    ap.add_argument("--temperature", type=float, default=None)
    ap.add_argument("--top-k", type=int, default=None)
    ap.add_argument("--output-format", choices=("auto", "decoded_text", "token_ids"), default=None)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--weights-url", default=None,
                    help="base URL (http(s):// or file://) of burnpack weights: resolved from the local cache "
                         "or fetched into it (parts first), then loaded in place of the run's checkpoint")
    ap.add_argument("--weights-cache", default=None, help="cache root for --weights-url (default: "
                    "$BURN_DRAGON_CACHE_DIR or ~/.cache/burn_dragon/models)")
    a = ap.parse_args(argv)
    run = RunDir(a.run)
    cfg = training_config_from_dict(run.read_json("training_config.json"))
    g = cfg.generation
    pick = lambda flag, conf: conf if flag is None else flag  # noqa: E731
    prompt_text = pick(a.prompt, g.prompt)
    max_tokens = pick(a.max_tokens, g.max_tokens)
    max_chars = pick(a.max_chars, g.max_chars)
    temperature = pick(a.temperature, g.temperature)
    top_k = pick(a.top_k, g.top_k)
    fmt = pick(a.output_format, g.output_format)
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    model = BDH(cfg.model, device=dev)
    if a.weights_url:
        from ..train import burnpack as BP
        from ..train.checkpoint import load_model_burnpack

        name = a.weights_url.rstrip("/").rpartition("/")[2]
        name = name[:-4] if name.endswith(".bpk") else name
        path = BP.resolve_or_bootstrap(name, a.weights_url, cache_root=a.weights_cache)
        load_model_burnpack(model, path)
    elif run.latest() is not None:
        run.load(None, model)
    tp = os.path.join(a.run, "tokenizer.json")
    run_tok = load_tokenizer(tp) if os.path.exists(tp) else load_tokenizer({"type": "byte"})

    def pick_tok(src: dict):
        if src.get("source", "dataset") == "dataset":
            return run_tok
        if src.get("path"):
            return load_tokenizer(src["path"])
        return load_tokenizer({k: v for k, v in src.items() if k not in ("source", "cache_dir")})

    tok, out_tok = pick_tok(g.prompt_tokenizer), pick_tok(g.decode_tokenizer)
    prompt = tok.encode(prompt_text) or [0]
    window = g.sliding_window(cfg.training.block_size)
    if window is not None and len(prompt) > window:
        prompt = prompt[-window:]  # the recurrent state carries the rest; nothing to trim later
    x = torch.tensor([prompt] * a.batch, dtype=torch.long, device=dev)
    out = Generator(model).generate(x, max_tokens, temperature=temperature, top_k=top_k, seed=a.seed)
    for row in out.tolist():
        if fmt == "token_ids":
            print(json.dumps(row))
        else:
            text = out_tok.decode(prompt + row)
            print(text[:len(prompt_text) + max_chars] if max_chars is not None else text)

if __name__ == "__main__":
    main()

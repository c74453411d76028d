"""Recurrent decode benchmark (the stateful-decode workload of the BDH-GPU configs).

  python -m burn_dragon_b200.cli.bench_decode [--batch 128] [--prompt 4096] [--tokens 64]

BDH-GPU (d=256, n=32768, h=4, L=6, RoPE), random-init weights, seeded random-byte
prompt. Prefill runs the fused inference forward in 512-token chunks carrying the state;
decode runs one token per sequence per step (greedy). Both phases are timed with CUDA
events after a warm-up; prints one JSON line (tokens/s over the whole batch).
"""

from __future__ import annotations

import argparse
import json

import torch

from ..config import DragonConfig
from ..models.bdh import BDH
from ..models.generate import Generator, sample_next
from ..ops.gemm import check_errors


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--prompt", type=int, default=4096)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--layers", type=int, default=6)
    ap.add_argument("--state-dtype", default="fp32", choices=["fp32", "bf16"])
    a = ap.parse_args()
    cfg = DragonConfig.bdh_gpu()
    cfg.n_layer = a.layers
    dev = torch.device("cuda", 0)
    model = BDH(cfg, device=dev, seed=1)
    g = Generator(model, prefill_chunk=512, state_dtype=a.state_dtype)
    gen = torch.Generator(device="cpu").manual_seed(20260729)
    prompt = torch.randint(0, 256, (a.batch, a.prompt), generator=gen).to(dev)
    # warm-up (compiles nothing; touches every kernel once)
    _, st = g.prefill(prompt[:, :512])
    g.decode_step(torch.zeros(a.batch, dtype=torch.long, device=dev), st)
    torch.cuda.synchronize()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record()
    logits, st = g.prefill(prompt)
    e[1].record()
    nxt = sample_next(logits)
    e[2].record()
    for _ in range(a.tokens):
        logits = g.decode_step(nxt, st)
        nxt = sample_next(logits)
    e[3].record()
    torch.cuda.synchronize()
    check_errors(dev)
    pre_ms = e[0].elapsed_time(e[1])
    dec_ms = e[2].elapsed_time(e[3])
    state_bytes = cfg.n_layer * a.batch * cfg.n_head * cfg.latent_per_head * cfg.n_embd * \
        (2 if a.state_dtype == "bf16" else 4)
    print(json.dumps({
        "metric": "recurrent decode tokens/s (device-timed) BDH-GPU",
        "batch": a.batch, "prompt": a.prompt, "decode_tokens": a.tokens, "state_dtype": a.state_dtype,
        "prefill_tokens_per_s": round(a.batch * a.prompt / (pre_ms / 1e3), 1),
        "decode_tokens_per_s": round(a.batch * a.tokens / (dec_ms / 1e3), 1),
        "decode_ms_per_token": round(dec_ms / a.tokens, 3),
        "state_bytes": state_bytes,
        "state_rw_gbs": round(2 * state_bytes / (dec_ms / a.tokens / 1e3) / 1e9, 1),
    }))


if __name__ == "__main__":
    main()

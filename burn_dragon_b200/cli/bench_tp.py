"""Tensor-parallel training benchmark for the 0.8B BDH config.

  python -m torch.distributed.run --nproc-per-node 8 -m burn_dragon_b200.cli.bench_tp

Config: d=1024, n=262144, h=8, L=8 shared layers, byte vocab, T=2048, global batch 64
of seeded random bytes, bf16 operands, AdamW; encoder / encoder_v / decoder sharded
along the neuron axis (one head per rank at 8 GPUs); gradient accumulation over
``--micro`` micro-batches to bound activation memory. Device-timed, max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

from ..config import DragonConfig
from ..train.data import RandomBytes
from ..train.trainer import Trainer, init_distributed


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--batch", type=int, default=64, help="global batch (replicated over TP ranks)")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--micro", type=int, default=8, help="micro-batches per step")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--dim", type=int, default=1024)
    ap.add_argument("--neurons", type=int, default=262144)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--sequence-parallel", action="store_true",
                    help="shard the residual stream by token rows between the tensor-parallel regions")
    a = ap.parse_args()
    rank, world, local = init_distributed()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = DragonConfig(n_layer=a.layers, n_embd=a.dim, n_head=a.heads, mlp_internal_dim_multiplier=a.neurons // a.dim,
                       dropout=0.0, rotary_embedding="rope")
    tr = Trainer(cfg, dev, lr=1e-3, seed=7, tensor_parallel=world > 1, micro_batches=a.micro,
                 sequence_parallel=a.sequence_parallel and world > 1)
    data = RandomBytes(a.batch, a.seq, seed=20260729)  # identical on every TP rank
    x, y = (t.to(dev) for t in data.next())
    for _ in range(a.warmup):
        tr.step(x, y)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        loss = tr.step(x, y)
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / a.steps], device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    if rank == 0:
        # roofline: each rank runs 1/W of the neuron-axis work (the embedding, norms, head and
        # CE are replicated and counted in full), and per layer and micro-batch the decoder
        # sum (forward) and the residual-gradient sum (backward) each reduce-scatter and
        # all-gather an fp32 [M, D] block: 4 (W - 1) / W * M * D * 4 bytes per direction
        from ..models.bdh_fused import STORES_X
        from ..train.roofline import measured_peaks, step_totals

        pk = measured_peaks()
        mb = a.batch // a.micro
        rows = step_totals(cfg, mb, a.seq, store_x=STORES_X, peaks=pk)["rows"]
        shared = ("embed + LN", "lm head", "cross-entropy", "d lm head (weight + input)", "AdamW")
        flop = sum(r["flop"] / (1 if r["kernel"] in shared else world) for r in rows) * a.micro
        link = 4 * a.layers * (world - 1) / world * mb * a.seq * a.dim * 4 * a.micro
        t_flop = flop / (pk["bf16_tflops_sustained"] * 1e12)
        t_link = link / 770e9
        step_s = ms.item() / 1e3
        toks = a.batch * a.seq
        print(json.dumps({"metric": "train tokens/sec (device-timed, max over ranks) BDH 0.8B neuron-TP",
                          "value": round(toks / (ms.item() / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
                          "ms_per_step": round(ms.item(), 2), "loss": float(loss.item()),
                          "per_gpu_tflop_per_step": round(flop / 1e12, 3),
                          "achieved_tflops_per_gpu": round(flop / step_s / 1e12, 1),
                          "nvlink_gb_per_direction_per_step": round(link / 1e9, 2),
                          "roofline_ms": round(max(t_flop, t_link) * 1e3, 1),
                          "frac_roofline": round(max(t_flop, t_link) / step_s, 3),
                          "peaks": {"bf16_tflops_sustained": pk["bf16_tflops_sustained"], "nvlink_gbs": 770.0,
                                    "source": pk["source"]},
                          "config": {"d": a.dim, "n": a.neurons, "h": a.heads, "L": a.layers, "T": a.seq,
                                     "global_batch": a.batch, "micro_batches": a.micro, "parallelism": f"tp{world}",
                                     "sequence_parallel": a.sequence_parallel}}),
              flush=True)
    if world > 1:
        dist.barrier()
    sys.stdout.flush()
    os._exit(0)


if __name__ == "__main__":
    main()

"""Pipeline-parallel training benchmark (fused stages, NCCL p2p between them).

  python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
      -m burn_dragon_b200.cli.bench_pipeline [--micro 8] [--schedule 1f1b]

BDH-GPU (d=256, n=32768, h=4, RoPE) with ``layers`` layers split over N stages, T=512,
``batch`` sequences per step in ``micro`` micro-batches, seeded random bytes, random-init
weights. Each rank runs its stage's fused forward / backward; activations and their
gradients move by NCCL isend / irecv posted ahead of the compute that needs them; the
gradients of the shared weights are summed over the stages, then AdamW. Times ``steps``
steps with CUDA events (max over ranks) and prints one JSON line.
"""

from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..config import DragonConfig
from ..models.bdh import BDH
from ..ops.gemm import check_errors
from ..parallel.pipeline import PipelineRunner, plan
from ..train.data import RandomBytes
from ..train.optim import FusedAdamW
from ..train.trainer import init_distributed


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--micro", type=int, default=8)
    ap.add_argument("--schedule", default="1f1b", choices=["gpipe", "1f1b"])
    a = ap.parse_args()
    rank, world, local = init_distributed()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = DragonConfig.bdh_gpu()
    cfg.n_layer = a.layers
    model = BDH(cfg, device=dev, seed=1337)
    opt = FusedAdamW(model.store, lr=1e-3, weight_decay=0.1)
    runner = PipelineRunner(model, plan(a.layers, world, a.micro, a.schedule), rank, a.batch // a.micro, a.seq)
    data = RandomBytes(a.batch, a.seq, seed=20260729)  # the same batch on every stage
    x, y = (t.to(dev) for t in data.next())

    def step():
        loss = runner.step(x, y)
        opt.step()
        return loss

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    loss = None
    for _ in range(a.steps):
        loss = step()
    e1.record()
    torch.cuda.synchronize()
    check_errors(dev)
    ms = torch.tensor([e0.elapsed_time(e1) / a.steps], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    lv = torch.tensor([float(loss) if loss is not None else 0.0], device=dev)
    dist.all_reduce(lv, op=dist.ReduceOp.MAX)
    if rank == 0:
        toks = a.batch * a.seq
        print(json.dumps({"metric": "train tokens/sec (device-timed, max over ranks) BDH-GPU pipeline",
                          "value": round(toks / (ms.item() / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
                          "ms_per_step": round(ms.item(), 3), "loss": float(lv.item()),
                          "config": {"layers": a.layers, "stages": world, "micro_batches": a.micro,
                                     "schedule": a.schedule, "batch": a.batch, "seq_len": a.seq}}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

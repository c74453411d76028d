"""Stateful-TBPTT training benchmark (the long-context BDH-GPU configuration).

  python -m burn_dragon_b200.cli.bench_tbptt [--batch 16] [--stream 8192] [--chunk 512]
  python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
      -m burn_dragon_b200.cli.bench_tbptt          (data parallel: N x batch streams)

BDH-GPU (d=256, n=32768, h=4, L=6, RoPE), random-init weights, seeded random-byte
streams. Every step trains the next ``chunk`` tokens of each stream with the recurrent
state carried (detached) from the previous chunk — the fused forward takes the state as
rho0 and returns the new one — and AdamW updates the weights. After a warm-up over one
full stream, one full stream (stream / chunk steps) is timed with CUDA events (max over ranks); prints
one JSON line (tokens/s over all ranks' streams). With N ranks every rank trains its own
``batch`` streams and the gradients meet in the NVLink data-parallel step.
"""

from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..config import DragonConfig
from ..models.state import ModelState
from ..ops.gemm import check_errors
from ..train.trainer import Trainer, init_distributed


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--stream", type=int, default=8192)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--layers", type=int, default=6)
    a = ap.parse_args()
    rank, world, local = init_distributed()
    torch.cuda.set_device(local)
    cfg = DragonConfig.bdh_gpu()
    cfg.n_layer = a.layers
    dev = torch.device("cuda", local)
    tr = Trainer(cfg, dev, lr=1e-3, weight_decay=0.0, comm="nvlink" if world > 1 else None)
    gen = torch.Generator().manual_seed(20260729 + 7919 * rank)
    data = torch.randint(0, 256, (a.batch, a.stream + 1), generator=gen).pin_memory()
    steps = a.stream // a.chunk

    def one_stream():
        st = ModelState.empty()
        loss = None
        for k in range(steps):
            s = k * a.chunk
            loss = tr.step_stream(data[:, s:s + a.chunk], data[:, s + 1:s + a.chunk + 1], st)
        return loss

    one_stream()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    loss = one_stream()
    e1.record()
    torch.cuda.synchronize()
    check_errors(dev)
    ms_t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    if rank == 0:
        # the carried state adds three contractions per layer (state read, state update and
        # its backward): the plain step's FLOPs at the same batch and their share explain
        # the per-token gap to plain training
        from ..models.bdh_fused import STORES_X
        from ..train.roofline import step_totals

        full = step_totals(cfg, a.batch, a.chunk, params=tr.model.store.numel, store_x=STORES_X, stateful=True)
        plain = step_totals(cfg, a.batch, a.chunk, params=tr.model.store.numel, store_x=STORES_X)
        step_s = ms / steps / 1e3
        print(json.dumps({
            "metric": "stateful TBPTT train tokens/s (device-timed, max over ranks) BDH-GPU",
            "n_gpus": world, "batch_per_gpu": a.batch, "stream": a.stream, "chunk": a.chunk, "steps": steps,
            "tokens_per_s": round(world * a.batch * a.stream / (ms / 1e3), 1),
            "ms_per_chunk_step": round(ms / steps, 3), "final_loss": float(loss),
            "chunk_step_tflop": round(full["tflop"], 3), "plain_step_tflop": round(plain["tflop"], 3),
            "state_flop_share": round(1 - plain["tflop"] / full["tflop"], 3),
            "achieved_tflops": round(full["tflop"] / step_s, 1),
            "frac_step_floor": round(full["floor_ms"] / (step_s * 1e3), 3),
        }), flush=True)
    if world > 1:
        if tr.comm is not None:
            tr.comm.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

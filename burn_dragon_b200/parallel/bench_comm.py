"""Microbenchmark of the data-parallel optimizer step over NVLink (one rank per GPU).

  python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
      -m burn_dragon_b200.parallel.bench_comm [--params 25300000] [--iters 50]

Times, with CUDA events on each rank and the max over ranks, (a) the whole NVLinkDDP
step (bf16 cast, barrier, fused reduce-scatter + AdamW + shadow all-gather, barrier),
(b) the same with global-norm clipping (``--transport nvls``: both through NVLink multicast
objects), and (c) the NCCL baseline: all-reduce (mean) of
the fp32 gradients followed by the fused AdamW on every rank. Reports the NVLink bytes
each rank moves and the achieved fraction of the roofline: (W-1)/W * P * 2 bytes in
each direction at 770 GB/s per direction (the measured peer-copy rate of this machine
class; 900 GB/s nominal).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _time(fn, iters: int, warmup: int = 5) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) * 1e3 / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--params", type=int, default=25_300_000)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--grad-dtype", default="bf16", choices=["bf16", "fp32"])
    ap.add_argument("--transport", default="p2p", choices=["p2p", "nvls"],
                    help="peer loads / stores, or NVLink multicast (in-switch sum, multicast stores)")
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl")
    rank, world = dist.get_rank(), dist.get_world_size()
    from .. import _ext
    from .ddp import NVLinkDDP

    class _Opt:  # the hyper-parameters NVLinkDDP.step_adamw reads
        b1, b2, eps, wd, clip = 0.9, 0.999, 1e-8, 0.1, None
        _hyper = torch.tensor([1e-3, 0.1, 0.001, 0.0], device="cuda")
        _scratch = torch.zeros(4, device="cuda")

    dev = torch.device("cuda", local)
    ddp = NVLinkDDP(a.params, dev, grad_dtype=a.grad_dtype, transport=a.transport)
    ddp.grad.normal_()
    ddp.param.normal_()
    opt = _Opt()
    us_step = _time(lambda: ddp.step_adamw(opt), a.iters)
    opt.clip = 1.0
    us_clip = _time(lambda: ddp.step_adamw(opt), a.iters)
    ddp.check()
    # NCCL baseline: fp32 all-reduce (mean) + full fused AdamW on every rank
    mod = _ext.load()
    g = torch.randn(ddp.numel, device="cuda")
    p = torch.randn(ddp.numel, device="cuda")
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    sh = torch.empty(ddp.numel, dtype=torch.bfloat16, device="cuda")

    def nccl_step():
        dist.all_reduce(g, op=dist.ReduceOp.AVG)
        mod.adamw(p, g, m, v, sh, 0.0, 0.9, 0.999, 1e-8, 0.1, 1.0, 1.0, None, opt._hyper)

    us_nccl = _time(nccl_step, a.iters)
    esz = 2 if a.grad_dtype == "bf16" else 4
    link_bytes = (world - 1) / world * ddp.numel * max(esz, 2)  # per direction, the larger of in / out
    roof_us = link_bytes / (LINK_GBS * 1e9) * 1e6
    if rank == 0:
        print(json.dumps({"world": world, "params": ddp.numel, "grad_dtype": a.grad_dtype, "transport": a.transport,
                          "nvlink_step_us": round(us_step, 1), "nvlink_step_clip_us": round(us_clip, 1),
                          "nccl_allreduce_adamw_us": round(us_nccl, 1),
                          "link_bytes_per_direction_mb": round(link_bytes / 1e6, 1),
                          "roofline_us": round(roof_us, 1),
                          "frac_roofline": round(roof_us / us_step, 3) if world > 1 else None}), flush=True)
    ddp.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

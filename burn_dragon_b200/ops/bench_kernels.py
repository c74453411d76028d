"""Microbenchmark of the non-GEMM kernels at the BDH-GPU training shapes, one case each.

  python -m burn_dragon_b200.ops.bench_kernels --case tail_fwd [--batch 32] [--iters 20]

Cases (B sequences of T = 512, D = 256, H = 4, Nh = 8192; M = B * T rows):
  ln_fwd        LayerNorm of a [M*H, D] fp32 attention output -> bf16
  ln_bwd        its backward, writing dC in [B, H, T, D] bf16 and gamma / beta partials
  tail_fwd      residual merge v' = LN(v + LN(sum of split-K partials)), fp32 + bf16 out
  tail_bwd      its backward
  symmetrize    G = mask(P) + mask(P)^T, [B*H, T, T] fp32 -> bf16
  adamw         fused AdamW over the 25.3M-parameter flat store (fp32 master, bf16 shadow)
  ddp_step      the NVLink data-parallel step's kernel at one rank (no peers: local reads
                and writes only; the 2..8-rank numbers come from parallel/bench_comm.py)
  scaffold_fold / scaffold_grad   the random-scaffold fold and adapter-gradient pass over
                the three projections (W_seed regenerated from the seed)
  rho_step      one decode step's state update + readout, batch = --batch (state fp32)
  ssd_fwd / ssd_bwd   the Mamba-3 chunk scan (BH = batch x 16 heads, T = 512, C = 64,
                S = 16, P = 128)
Prints one JSON line: device time per launch (CUDA events after warm-up), algorithmic
bytes and the achieved rate. Used to size ncu captures of a single kernel.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from .. import _ext


def build(case: str, B: int):
    mod = _ext.load()
    dev = "cuda"
    T, D, H, Nh = 512, 256, 4, 8192
    M, N = B * T, H * Nh
    f32, bf = torch.float32, torch.bfloat16
    r = lambda *s: torch.randn(*s, device=dev)  # noqa: E731
    gam, bet = 1 + 0.1 * r(D), 0.1 * r(D)
    if case == "ln_fwd":
        x, y16, mean, rstd = r(M * H, D), torch.empty(M * H, D, dtype=bf, device=dev), r(M * H), r(M * H)
        return (lambda: mod.ln_fwd(x, None, M * H, D, gam, bet, 1e-5, None, y16, mean, rstd)), M * H * D * 6
    if case == "ln_bwd":
        dy, x, mean, rstd = r(M, H, D), r(M, H, D), r(M * H), r(M * H).abs() + 0.5
        dC = torch.empty(B, H, T, D, dtype=bf, device=dev)
        return (lambda: mod.ln_bwd(dy, x, mean, rstd, M * H, D, gam, T, H, dC, None)), M * H * D * 10
    if case == "tail_fwd":
        splits = 2
        part, v = r(splits, M, D), r(M, D)
        m, o32, o16, st = torch.empty(M, D, device=dev), torch.empty(M, D, device=dev), \
            torch.empty(M, D, dtype=bf, device=dev), torch.empty(M, 4, device=dev)
        return (lambda: mod.tail_fwd(part, splits, M * D, v, M, D, gam, bet, 1e-5, m, o32, o16, st)), \
            M * D * (4 * splits + 4 + 4 + 4 + 2)
    if case == "tail_bwd":
        g, v, m, st = r(M, D), r(M, D), r(M, D), r(M, 4).abs() + 0.5
        dm16, dres = torch.empty(M, D, dtype=bf, device=dev), torch.empty(M, D, device=dev)
        return (lambda: mod.tail_bwd(g, v, m, st, M, D, gam, bet, dm16, dres)), M * D * (4 * 3 + 2 + 4)
    if case == "symmetrize":
        P, G = r(B * H, T, T), torch.empty(B * H, T, T, dtype=bf, device=dev)
        return (lambda: mod.symmetrize(P, G, B * H, T, H, None)), B * H * T * T * 6
    if case in ("adamw", "ddp_step"):
        n = 25_300_032
        p, g, m, v = r(n), r(n), torch.zeros(n, device=dev), torch.zeros(n, device=dev)
        sh = torch.empty(n, dtype=bf, device=dev)
        hyper = torch.tensor([1e-3, 0.1, 0.001, 0.0], device=dev)
        if case == "adamw":
            return (lambda: mod.adamw(p, g, m, v, sh, 0.0, 0.9, 0.999, 1e-8, 0.1, 1.0, 1.0, None, hyper)), n * 30
        g16 = g.to(bf)
        gp, sp = [g16.data_ptr()], [sh.data_ptr()]
        return (lambda: mod.ddp_step(gp, sp, True, 0, 0, n, p, m, v, 0.9, 0.999, 1e-8, 0.1, hyper, None, [])), n * 28
    if case in ("scaffold_fold", "scaffold_grad"):
        from ..config import DragonConfig, RandomScaffoldConfig
        from ..models.bdh import BDH
        from ..models.scaffold import base_shape

        cfg = DragonConfig.bdh_gpu()
        cfg.random_scaffold = RandomScaffoldConfig(enabled=True, seed=20260729, rank=16, alpha=16.0,
                                                   scaling="rank_stabilized", trainable_gain=True)
        model = BDH(cfg, device=dev, seed=1)
        nel = sum(torch.Size(base_shape(cfg, k)).numel() for k in ("encoder", "encoder_v", "decoder"))
        if case == "scaffold_fold":
            p16, g32 = model.shadow_dict(), model.grad_dict()
            return (lambda: model._scaffold_prepare(p16, g32)), nel * 2
        p16, g32 = model.shadow_dict(), model.grad_dict()
        model._scaffold_prepare(p16, g32)
        for t in model._geff.values():
            t.normal_()
        return (lambda: model._scaffold_backward(g32)), nel * 4
    if case == "rho_step":
        rho, q, v = r(B, H, Nh, D), torch.relu(r(B, N)).to(bf), r(B, D)
        a = torch.zeros(B, H, D, device=dev)
        return (lambda: mod.rho_step(rho, q, N, v, None, a, B, H, Nh, D)), rho.numel() * 8
    if case in ("ssd_fwd", "ssd_bwd"):
        BH, C, S, P = B * 16, 64, 16, 128
        n = T // C
        q, k, v = r(BH, T, S) * 0.3, r(BH, T, S) * 0.3, r(BH, T, P)
        da = torch.cat([c.cumsum(1) for c in (-0.01 * torch.rand(BH, T, device=dev)).split(C, 1)], 1).contiguous()
        s0, vs, ks, cf = r(BH, P, S), r(BH, n, P), r(BH, n, S), torch.rand(BH, n, device=dev)
        y, sf, sc = torch.empty(BH, T, P, device=dev), torch.empty(BH, P, S, device=dev), \
            torch.empty(BH, n, P, S, device=dev)
        io = (2 * BH * T * S + 2 * BH * T * P + BH * n * P * S) * 4
        if case == "ssd_fwd":
            return (lambda: mod.ssd_chunk_fwd(q, k, v, da, s0, vs, ks, cf, C, y, sf, sc)), io
        mod.ssd_chunk_fwd(q, k, v, da, s0, vs, ks, cf, C, y, sf, sc)
        dy, dsf = r(BH, T, P), r(BH, P, S)
        outs = [torch.empty_like(t) for t in (q, k, v, da)] + [torch.empty_like(s0), torch.empty_like(vs),
                                                              torch.empty_like(ks), torch.empty_like(cf)]
        return (lambda: mod.ssd_chunk_bwd(q, k, v, da, vs, ks, cf, sc, dy, dsf, C, *outs)), 2 * io
    raise ValueError(case)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    call, nbytes = build(a.case, a.batch)
    for _ in range(a.warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        call()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / a.iters
    print(json.dumps({"case": a.case, "batch": a.batch, "us": round(us, 1), "bytes": nbytes,
                      "gbs": round(nbytes / us / 1e3, 1), "pid": os.getpid()}))


if __name__ == "__main__":
    main()

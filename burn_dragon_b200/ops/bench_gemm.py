"""Microbenchmark of the BDH contractions on the tcgen05 engine, one case at a time.

  python -m burn_dragon_b200.ops.bench_gemm --case dq --batch 4 [--iters 20]

Each case builds the operands with the exact layouts the fused BDH step uses (d=256,
h=4, Nh=8192, T=512 unless overridden) and reports device time (CUDA events, after
warm-up), achieved TFLOP/s and the algorithmic HBM bytes / time. Used to size and
drive ncu captures of a single kernel on a small case.
"""

from __future__ import annotations

import argparse
import os
import json

import torch

from . import gemm as G
from .gemm import Operand


def build(case: str, B: int, T: int, D: int, H: int, Nh: int):
    dev = "cuda"
    N, M = H * Nh, B * T
    bf = torch.bfloat16
    r = lambda *s: (torch.randn(*s, device=dev) * 0.5).to(bf)  # noqa: E731
    freq = torch.rand(Nh, device=dev) * 0.1
    if os.environ.get("BDH_BENCH_NOROPE"):
        freq = None  # the epilogue without the rotation (cost split of the RoPE math)
    tab = None
    if freq is not None and os.environ.get("BDH_BENCH_ROPE_TABLE", "0") == "1":
        tab = G.rope_table(freq, 0, T)  # the half2 phase table the fused step passes
    if case == "xproj":
        v, enc, x, q = r(M, D), r(H, D, Nh), r(M, N), r(M, N)
        call = lambda: G.gemm(G.EPI_RELU_ROPE, Operand(v, False, D, M, D),  # noqa: E731
                              Operand(enc, True, Nh, D, Nh, z1=(H, D * Nh)), M, Nh, D, x, Z1=H, bn=G.tma_bn(M, Nh), out1=q, ld=N,
                              sz1=Nh, freq=freq, T=T, Nh=Nh, rope_tab=tab)
        return call, 2 * M * N * D, (M * D + D * N + 2 * M * N) * 2
    if case == "scores":
        q, S = r(M, N), r(B, H, T, T)
        op = Operand(q, False, Nh, T, N, z1=(H, Nh), z2=(B, T * N))
        bn = int(os.environ.get("BDH_BENCH_BN", "256"))
        call = lambda: G.gemm(G.EPI_SCORES, op, op, T, T, Nh, S, Z1=H, Z2=B, bn=bn, causal_skip=True,  # noqa: E731
                              ld=T, sz1=T * T, sz2=H * T * T)
        return call, B * H * T * T * Nh, (M * N + B * H * T * T) * 2
    if case == "gate":
        an, encv, x, yn = r(M, H, D), r(H, D, Nh), r(M, N), r(M, N)
        call = lambda: G.gemm(G.EPI_GATE, Operand(an, False, D, M, H * D, z1=(H, D)),  # noqa: E731
                              Operand(encv, True, Nh, D, Nh, z1=(H, D * Nh)), M, Nh, D, yn, Z1=H, bn=G.tma_bn(M, Nh), aux0=x, ld=N,
                              sz1=Nh)
        return call, 2 * M * N * D, (M * H * D + D * N + 2 * M * N) * 2
    if case == "dec_bwd":
        dm, dec, x, yn, dx, dy = r(M, D), r(N, D), r(M, N), r(M, N), r(M, N), r(M, N)
        call = lambda: G.gemm(G.EPI_DEC_BWD, Operand(dm, False, D, M, D), Operand(dec, False, D, N, D),  # noqa: E731
                              M, N, D, dx, bn=G.tma_bn(M, N), out1=dy, aux0=x, aux1=yn, ld=N)
        return call, 2 * M * N * D, (M * D + N * D + 4 * M * N) * 2
    if case == "dq":
        g16, q, dx = r(B, H, T, T), r(M, N), r(M, N)
        call = lambda: G.gemm(G.EPI_DQ, Operand(g16, False, T, T, T, z1=(H, T * T), z2=(B, H * T * T)),  # noqa: E731
                              Operand(q, True, Nh, T, N, z1=(H, Nh), z2=(B, T * N)), T, Nh, T, dx, Z1=H, Z2=B, bn=G.tma_bn(T, Nh, "dq"),
                              aux0=dx, ld=N, sz1=Nh, sz2=T * N, freq=freq, T=T, Nh=Nh, rope_tab=tab)
        return call, 2 * B * H * T * T * Nh, (B * H * T * T + 3 * M * N) * 2
    if case == "wgrad":
        a, dy, out = r(M, D), r(M, N), torch.zeros(H, D, Nh, device=dev)
        call = lambda: G.gemm(G.EPI_F32, Operand(a, True, D, M, D), Operand(dy, True, Nh, M, N, z1=(H, Nh)),  # noqa: E731
                              D, Nh, M, out, Z1=H, ld=Nh, sz1=D * Nh, accumulate=True)
        return call, 2 * M * N * D, (M * D + M * N) * 2 + 2 * D * N * 4
    if case == "dec_fwd":
        yn, dec = r(M, N), r(N, D)
        kb = N // 64
        splits = G.fit_splits(kb, max(1, -(-2 * 148 // (M // 128))))
        part = torch.empty(splits, M, D, device=dev)
        call = lambda: G.gemm(G.EPI_F32, Operand(yn, False, N, M, N), Operand(dec, True, D, N, D), M, D, N,  # noqa: E731
                              part, splits=splits, ld=D, split_stride=M * D)
        return call, 2 * M * N * D, M * N * 2 + splits * M * D * 4
    if case == "k256":
        # the x-projection's operands with a plain bf16 output (no ReLU / RoPE, one tensor)
        v, enc, x = r(M, D), r(H, D, Nh), r(M, N)
        call = lambda: G.gemm(G.EPI_BF16, Operand(v, False, D, M, D),  # noqa: E731
                              Operand(enc, True, Nh, D, Nh, z1=(H, D * Nh)), M, Nh, D, x, Z1=H, bn=128, ld=N, sz1=Nh)
        return call, 2 * M * N * D, (M * D + D * N + M * N) * 2
    if case == "plain":
        # square K-major GEMM with an fp32 output: tile shape / CTA-pair comparison
        # (BDH_BENCH_BN, BDH_BENCH_PAIR); M = N = batch * 1024, K = seq * 16
        Mp, Kp = B * 1024, T * 16
        a, b, out = r(Mp, Kp), r(Mp, Kp), torch.empty(Mp, Mp, device=dev)
        bn = int(os.environ.get("BDH_BENCH_BN", "256"))
        pair = os.environ.get("BDH_BENCH_PAIR", "1") != "0"
        call = lambda: G.gemm(G.EPI_F32, Operand(a, False, Kp, Mp, Kp), Operand(b, False, Kp, Mp, Kp),  # noqa: E731
                              Mp, Mp, Kp, out, bn=bn, ld=Mp, pair=pair)
        return call, 2 * Mp * Mp * Kp, (2 * Mp * Kp) * 2 + Mp * Mp * 4
    raise ValueError(case)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--dim", type=int, default=256)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--latent", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    call, flops, nbytes = build(a.case, a.batch, a.seq, a.dim, a.heads, a.latent)
    for _ in range(a.warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        call()
    e1.record()
    torch.cuda.synchronize()
    G.check_errors(torch.device("cuda"))
    us = e0.elapsed_time(e1) * 1e3 / a.iters
    print(json.dumps({"case": a.case, "batch": a.batch, "us": round(us, 1), "tflops": round(flops / us / 1e6, 1),
                      "gbs": round(nbytes / us / 1e3, 1)}))


if __name__ == "__main__":
    main()

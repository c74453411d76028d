"""Step-level roofline of the fused BDH training step: FLOPs and HBM bytes per kernel.

``fused_step_cost(cfg, B, T)`` lists every contraction and row kernel that one fused
training step (forward, CE, backward, AdamW) launches, with

* ``flop``: the algorithmic multiply-add work (2 per MAC) the kernel must do. Causal
  products count the strictly-lower triangle only (the engine skips tiles above the
  diagonal; tiles on it are computed in full, which the ``flop_exec`` column adds).
* ``bytes``: the HBM traffic of the design: every operand that is not L2-resident read
  once, every output written once. The weights (a few MB) and the per-head [T, T]
  blocks that the next kernel re-reads from L2 are counted once.

The sums give the step's floor: ``max(flop / bf16 peak, bytes / HBM bandwidth)`` per
kernel, added over kernels (kernels run one after another). Peaks are the measured
figures of the machine (``measured_peaks()``), with fixed fallbacks.

The reference logs only the forward's four contraction terms
(burn_dragon_language/src/train/utils.rs:130-154); ``train.metrics.theoretical_forward_flops``
restates that log. This table is the per-kernel breakdown of the step this package runs.
"""

from __future__ import annotations

import json
import os

# Fallback denominators (a plain copy and a cuBLAS bf16 GEMM on a B200 of this pool).
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def measured_peaks(path: str | None = None) -> dict:
    """The measured copy bandwidth (GB/s) and bf16 GEMM rate (TFLOP/s, burst and
    sustained) from ``MEASURED_PEAKS.json`` at the repository root, else the fallback.
    The returned dict says which (``source``)."""
    if path is None:
        path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                            "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        out = {k: float(d[k]) for k in FALLBACK}
        out["source"] = "measured"
        return out
    except (OSError, KeyError, ValueError, TypeError):
        out = dict(FALLBACK)
        out["source"] = "fallback"
        return out


def fused_step_cost(cfg, B: int, T: int, store_x: bool = False, stateful: bool = False) -> list[dict]:
    """Per-kernel FLOPs / bytes of one fused step at batch ``B`` x ``T`` tokens.

    ``store_x``: the forward also stores x next to q (an older layout); by default x is
    recovered from q = rope(x) and a one-bit positivity mask where it is read.
    ``stateful``: a TBPTT chunk step, which also reads the carried state rho0 [B,H,Nh,D]
    (a += q rho0, dq += dC rho0^T) and writes the outgoing one (rho_T = q^T v + rho0)."""
    D, H, Nh, V, L = cfg.n_embd, cfg.n_head, cfg.latent_per_head, cfg.vocab_size, cfg.n_layer
    N = H * Nh
    M = B * T
    bf, f4 = 2, 4
    MN = M * N * bf           # one bf16 [M, N] activation
    MD4 = M * D * f4          # one fp32 [M, D] stream
    MD2 = M * D * bf
    mask = M * N // 8         # one bit per neuron activation
    tri = T * (T - 1) // 2    # strictly-causal pairs per sequence
    diag_extra = (T // 128) * 128 * 129 // 2  # computed-in-full diagonal-tile entries (engine)
    S = B * H * T * T * bf    # bf16 scores
    P = B * H * T * T * f4
    rows = []

    def k(name, flop, byts, per_layer=True, flop_exec=None):
        rows.append({"kernel": name, "flop": flop * (L if per_layer else 1),
                     "flop_exec": (flop_exec if flop_exec is not None else flop) * (L if per_layer else 1),
                     "bytes": byts * (L if per_layer else 1)})

    mnd = 2 * M * N * D
    q_w = MN + (MN if store_x else mask)
    # ---- forward
    k("embed + LN", 0, M * 8 + 2 * MD4 + MD2, per_layer=False)
    k("x-projection + ReLU + RoPE", mnd, MD2 + q_w)
    k("causal scores q q^T", 2 * B * H * tri * Nh, MN + S, flop_exec=2 * B * H * (tri + diag_extra) * Nh)
    k("S V", 2 * B * H * tri * D, S + MD2 + M * H * D * f4)
    k("LayerNorm(a)", 0, M * H * D * (f4 + bf))
    k("gate y = relu(an Dy) * x", mnd, M * H * D * bf + (MN if store_x else MN + mask) + MN)
    k("decoder yn E (split-K)", mnd, MN + 2 * MD4)
    k("residual merge (tail)", 0, 2 * MD4 + MD4 + MD2 + MD4)
    k("lm head", 2 * M * D * V, MD2 + M * V * f4, per_layer=False)
    k("cross-entropy", 0, M * V * (f4 + bf), per_layer=False)
    # ---- backward
    k("d lm head (weight + input)", 4 * M * D * V, 2 * M * V * bf + MD2 + MD4, per_layer=False)
    k("tail backward", 0, 3 * MD4 + MD2 + MD4)
    k("decoder backward d(yn) -> dx_part, dy_pre", mnd, MD2 + (MN if store_x else MN + mask) + MN + 2 * MN)
    k("dE += yn^T dm", mnd, MN + MD2)
    k("dDy += an^T dy", mnd, MN + M * H * D * bf)
    k("d(an) = dy Dy^T", mnd, MN + M * H * D * f4)
    k("LayerNorm backward -> dC", 0, M * H * D * (2 * f4 + bf))
    k("P = dC V^T", 2 * B * H * tri * D, M * H * D * bf + MD2 + P)
    k("symmetrize G = dS + dS^T", 0, P + S)
    k("dQ: (dx_part + rope^T(G q)) masked", 2 * B * H * T * T * Nh, S + MN + MN + MN)
    k("dV = sum_h S^T dC", 2 * B * H * tri * D, S + M * H * D * bf + MD4)
    k("dDx += v^T dx", mnd, MN + MD2)
    k("dv_x = dx Dx^T (per head)", mnd, MN + H * MD4)
    k("dv sum", 0, (H + 3) * MD4)
    if stateful:
        R4, R2 = B * H * Nh * D * f4, B * H * Nh * D * bf
        k("state read a += q rho0", 2 * B * H * T * Nh * D, MN + R2 + M * H * D * f4 * 2)
        k("state update rho_T = q^T v + rho0", 2 * B * H * Nh * T * D, MN + MD2 + R4 + R4 + R2)
        k("state backward dq += rope^T(dC rho0^T)", 2 * B * H * T * D * Nh, M * H * D * bf + R2 + MN + MN)
    k("AdamW", 0, 0, per_layer=False)
    return rows


def step_totals(cfg, B: int, T: int, params: int = 0, store_x: bool = False, peaks: dict | None = None,
                stateful: bool = False) -> dict:
    """Summed FLOPs / bytes of a step and the floor time at the given peaks.

    ``params``: parameter count (AdamW reads p, g, m, v and writes p, m, v, bf16 shadow)."""
    rows = fused_step_cost(cfg, B, T, store_x=store_x, stateful=stateful)
    for r in rows:
        if r["kernel"] == "AdamW":
            r["bytes"] = params * (4 * 4 + 3 * 4 + 2)
    pk = peaks or measured_peaks()
    flop = sum(r["flop"] for r in rows)
    byts = sum(r["bytes"] for r in rows)
    floor_s = 0.0
    for r in rows:
        floor_s += max(r["flop"] / (pk["bf16_tflops_sustained"] * 1e12), r["bytes"] / (pk["hbm_gbs"] * 1e9))
    return {"tflop": flop / 1e12, "hbm_gb": byts / 1e9, "floor_ms": floor_s * 1e3, "peaks": pk, "rows": rows}

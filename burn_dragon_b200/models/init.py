"""Weight initialisation schemes (burn_dragon_core/src/model/init.rs).

``initialization`` selects the family for the three shared projections, the embedding
and the LM head:

* ``simple_normal``: N(0, init_std) everywhere (the BASELINE configurations);
* ``near_critical`` (the reference's default): projection std
  ``min(1/sqrt(fan_in + fan_out), 0.02)`` (init.rs:857-859), embedding
  ``min(1/sqrt(width), 0.02)`` (init.rs:853-855), residual-branch projections (encoder,
  encoder_v, decoder) scaled by ``1/sqrt(residual_depth)`` (init.rs:398-405,625-650);
* ``he_glorot``: He std ``sqrt(2/fan_in)`` for the encoders, Glorot
  ``sqrt(2/(fan_in+fan_out))`` for decoder and head (init.rs:611-620,877-883);
* ``headwise_semi_orthogonal``: near-critical std, realised as block-orthonormal
  matrices scaled by ``std * sqrt(min(rows, cols))`` per head (init.rs:968-1010);
* ``reservoir``: near-critical RMS with a sparse (``reservoir_density``) Gaussian
  pattern rescaled to that RMS — this framework's reading of the reservoir family
  (the reference's topology priors are not reproduced).
"""

from __future__ import annotations

import math

import torch

CAP = 0.02


def near_critical_projection_std(fan_in: int, fan_out: int) -> float:
    return min(1.0 / math.sqrt(max(fan_in, 1) + max(fan_out, 1)), CAP)


def near_critical_embedding_std(width: int) -> float:
    return min(1.0 / math.sqrt(max(width, 1)), CAP)


def _semi_orthogonal(rows: int, cols: int, std: float, gen: torch.Generator) -> torch.Tensor:
    block = max(1, min(rows, cols))
    gain = std * math.sqrt(block)
    out = torch.empty(rows, cols)
    if rows <= cols:
        for c0 in range(0, cols, block):
            q, _ = torch.linalg.qr(torch.randn(block, block, generator=gen))
            w = min(block, cols - c0)
            out[:, c0:c0 + w] = q[:rows, :w] * gain
    else:
        for r0 in range(0, rows, block):
            q, _ = torch.linalg.qr(torch.randn(block, block, generator=gen))
            h = min(block, rows - r0)
            out[r0:r0 + h, :] = q[:h, :cols] * gain
    return out


def init_tensor(kind: str, role: str, shape, fan_in: int, fan_out: int, depth: int, gen: torch.Generator,
                init_std: float = 0.02, density: float = 0.1) -> torch.Tensor:
    """role: encoder | encoder_v | decoder | embed | lm_head."""
    residual = role in ("encoder", "encoder_v", "decoder")
    if kind == "simple_normal":
        return torch.randn(shape, generator=gen) * init_std
    if kind == "he_glorot":
        std = math.sqrt(2.0 / max(fan_in, 1)) if role in ("encoder", "encoder_v") else \
            math.sqrt(2.0 / (max(fan_in, 1) + max(fan_out, 1)))
        if role == "embed":
            std = near_critical_embedding_std(fan_out)
        return torch.randn(shape, generator=gen) * std
    if role == "embed":
        std = near_critical_embedding_std(fan_out)
    else:
        std = near_critical_projection_std(fan_in, fan_out)
        if residual:
            std /= math.sqrt(max(depth, 1))
    if kind == "near_critical" or role in ("embed",):
        return torch.randn(shape, generator=gen) * std
    if kind == "headwise_semi_orthogonal":
        if len(shape) == 3:
            return torch.stack([_semi_orthogonal(shape[1], shape[2], std, gen) for _ in range(shape[0])])
        return _semi_orthogonal(shape[0], shape[1], std, gen)
    if kind == "reservoir":
        w = torch.randn(shape, generator=gen)
        mask = (torch.rand(shape, generator=gen) < density).float()
        w = w * mask
        rms = w.pow(2).mean().sqrt().clamp_min(1e-12)
        return w * (std / rms)
    raise ValueError(f"unknown initialization kind {kind!r}")

"""Weight initialisation (burn_dragon_core/src/model/init.rs).

``initialization`` selects the family for the shared projections, the embedding and the
LM head, and ``init_param`` applies the reference's modifiers:

* base std: ``simple_normal`` = ``init_std``; ``near_critical`` (also the base of
  ``headwise_semi_orthogonal`` and ``reservoir``) = ``min(1/sqrt(fan_in + fan_out), 0.02)``
  (init.rs:857-859); ``he_glorot`` = He ``sqrt(2/fan_in)`` for the encoders, Glorot
  ``sqrt(2/(fan_in+fan_out))`` for decoder and head (init.rs:611-620,877-883);
* embedding std: near-critical ``min(1/sqrt(width), 0.02)``, ``init_std``, or Glorot
  ``sqrt(1/width)`` (init.rs:588-596);
* residual scaling of the three shared projections: ``family_default`` (1/sqrt(depth) for
  the near-critical family, else 1), ``disabled``, ``depth_scaled`` (1/sqrt(depth)), times
  ``residual_scaling_gain``; depth = n_layer * rollout fast steps (init.rs:620-650);
* ``headwise_semi_orthogonal``: block-orthonormal matrices scaled to the target std per
  head (init.rs:968-1010);
* neuron gains (``heavy_tailed_log_normal``): per output neuron of encoder / encoder_v
  ([H, Nh]) and per decoder row, ``exp(N(0, log_sigma))`` clipped at ``max_gain`` and
  normalised to unit RMS (init.rs:760-806);
* topology prior (``modular_bridges``): a fixed [fan_in, fan_out] multiplier — community
  blocks (intra / inter gain) plus a tail of "bridge" latent neurons — normalised to unit
  RMS, on the latent columns of the encoders and the latent rows of the decoder
  (init.rs:690-750,1076-1120);
* ``reservoir``: near-critical RMS with a sparse (``reservoir_density``) Gaussian pattern
  rescaled to that RMS — this framework's reading of the reservoir family (the
  reference's reservoir topology options are not reproduced); no gains or prior.
"""

from __future__ import annotations

import math

import torch

CAP = 0.02
NC_FAMILY = ("near_critical", "headwise_semi_orthogonal", "reservoir")


def near_critical_projection_std(fan_in: int, fan_out: int) -> float:
    return min(1.0 / math.sqrt(max(fan_in, 1) + max(fan_out, 1)), CAP)


def near_critical_embedding_std(width: int) -> float:
    return min(1.0 / math.sqrt(max(width, 1)), CAP)


def base_projection_std(cfg, role: str, fan_in: int, fan_out: int) -> float:
    k = cfg.initialization
    if k in NC_FAMILY:
        return near_critical_projection_std(fan_in, fan_out)
    if k == "simple_normal":
        return cfg.init_std
    if role in ("encoder", "encoder_v"):
        return math.sqrt(2.0 / max(fan_in, 1))
    return math.sqrt(2.0 / (max(fan_in, 1) + max(fan_out, 1)))


def residual_factor(cfg, role: str) -> float:
    if role not in ("encoder", "encoder_v", "decoder"):
        return 1.0
    kind = cfg.residual_scaling
    depth = cfg.residual_depth()
    if kind == "depth_scaled" or (kind == "family_default" and cfg.initialization in NC_FAMILY):
        f = 1.0 / math.sqrt(depth)
    else:
        f = 1.0
    return f * cfg.residual_scaling_gain


def projection_std(cfg, role: str, fan_in: int, fan_out: int) -> float:
    return base_projection_std(cfg, role, fan_in, fan_out) * residual_factor(cfg, role)


def embedding_std(cfg, width: int) -> float:
    k = cfg.initialization
    if k in NC_FAMILY:
        return near_critical_embedding_std(width)
    if k == "simple_normal":
        return cfg.init_std
    return math.sqrt(2.0 / (2 * max(width, 1)))


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


def neuron_gains(cfg, shape, gen: torch.Generator) -> torch.Tensor:
    if cfg.neuron_gains == "iid":
        return torch.ones(shape)
    g = (torch.randn(shape, generator=gen) * cfg.neuron_gain_log_sigma).exp().clamp(max=cfg.neuron_gain_max)
    return g / g.pow(2).mean().sqrt().clamp_min(1e-6)


def modular_bridges(cfg, rows: int, cols: int, latent_axis: str) -> torch.Tensor:
    """[rows, cols] community / bridge multiplier at unit RMS; ``latent_axis`` (rows or
    cols) is the axis whose last ``bridge_fraction`` indices are bridge neurons."""
    rows, cols = max(rows, 1), max(cols, 1)
    latent = rows if latent_axis == "rows" else cols
    bridges = min(int(round(latent * cfg.topology_bridge_fraction)), latent)
    comm = max(1, min(cfg.topology_community_count, min(rows, cols)))
    rc = (torch.arange(rows) * comm) // rows
    cc = (torch.arange(cols) * comm) // cols
    v = torch.where(rc[:, None] == cc[None, :], cfg.topology_intra_community_gain, cfg.topology_inter_community_gain)
    v = v.to(torch.float64)
    idx = torch.arange(latent) >= latent - bridges
    if latent_axis == "rows":
        v[idx, :] = cfg.topology_bridge_gain
    else:
        v[:, idx] = cfg.topology_bridge_gain
    return (v / v.pow(2).mean().sqrt().clamp_min(1e-12)).float()


def init_param(cfg, role: str, shape, gen: torch.Generator) -> torch.Tensor:
    """role: encoder | encoder_v ([H, D, Nh]) | decoder ([N, D]) | embed ([V, D]) |
    lm_head ([D, V])."""
    if role == "embed":
        return torch.randn(shape, generator=gen) * embedding_std(cfg, shape[1])
    if len(shape) == 3:
        fan_in, fan_out = shape[1], shape[2]
    else:
        fan_in, fan_out = shape[0], shape[1]
    std = projection_std(cfg, role, fan_in, fan_out)
    kind = cfg.initialization
    if kind == "reservoir" and role != "lm_head":
        w = torch.randn(shape, generator=gen)
        w = w * (torch.rand(shape, generator=gen) < cfg.reservoir_density).float()
        return w * (std / w.pow(2).mean().sqrt().clamp_min(1e-12))
    if kind == "headwise_semi_orthogonal" and role in ("encoder", "encoder_v"):
        w = torch.stack([_semi_orthogonal(fan_in, fan_out, std, gen) for _ in range(shape[0])])
    elif kind == "headwise_semi_orthogonal" and role == "decoder":
        w = _semi_orthogonal(fan_in, fan_out, std, gen)
    else:
        w = torch.randn(shape, generator=gen) * std
    if role in ("encoder", "encoder_v"):
        w = w * neuron_gains(cfg, (shape[0], 1, fan_out), gen)
        if cfg.topology_prior == "modular_bridges":
            w = w * modular_bridges(cfg, fan_in, fan_out, "cols")[None]
    elif role == "decoder":
        w = w * neuron_gains(cfg, (fan_in, 1), gen)
        if cfg.topology_prior == "modular_bridges":
            w = w * modular_bridges(cfg, fan_in, fan_out, "rows")
    return w


def init_tensor(kind: str, role: str, shape, fan_in: int, fan_out: int, depth: int, gen: torch.Generator,
                init_std: float = 0.02, density: float = 0.1) -> torch.Tensor:
    """Family-only draw (no residual-scaling sub-config, gains or prior): the
    ``family_default`` scaling with iid neurons."""
    from types import SimpleNamespace

    cfg = SimpleNamespace(initialization=kind, init_std=init_std, reservoir_density=density,
                          residual_scaling="family_default", residual_scaling_gain=1.0, neuron_gains="iid",
                          topology_prior="iid", residual_depth=lambda: max(depth, 1))
    if role == "embed":
        return torch.randn(shape, generator=gen) * embedding_std(cfg, fan_out)
    return init_param(cfg, role, shape, gen)

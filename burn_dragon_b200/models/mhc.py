"""Manifold-constrained hyper-connections (mHC), static-Sinkhorn policy
(burn_dragon_core/src/model/mhc/reference.rs:18-675).

The residual stream becomes S parallel streams R [B, S, T, D]. Per layer:
  H_res  = Sinkhorn(h_res / tau) (doubly stochastic S x S; iters of row / column
           log-softmax), initialised near the identity (diagonal 0, off-diagonal -8);
  H_pre  = softmax(h_pre, over streams) [V, S]: the branch input is the stream mixture
           sum_s H_pre[v, s] R_s (one view, V = 1);
  H_post = softmax(h_post, over streams) [V, S]: the branch output is distributed back,
  R <- H_res-mixed R + sum_v H_post[v, s] * branch_out_v.
The initial streams repeat the embedded input; the LM head reads the mean of the
streams. Only the PyTorch path implements mHC.
"""

from __future__ import annotations

import torch


def sinkhorn(logits: torch.Tensor, tau: float = 1.0, iters: int = 10) -> torch.Tensor:
    z = logits / max(tau, 1e-6)
    for _ in range(iters):
        z = torch.log_softmax(z, dim=-1)
        z = torch.log_softmax(z, dim=-2)
    return z.exp()


def mix(streams: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """streams [B, S_in, T, D], w [S_in, S_out] -> [B, S_out, T, D]."""
    return torch.einsum("bitd,io->botd", streams, w)


def init_logits(n_layer: int, streams: int, views: int = 1) -> dict[str, torch.Tensor]:
    res = torch.full((n_layer, streams, streams), -8.0)
    pre = torch.full((n_layer, views, streams), -8.0)
    post = torch.full((n_layer, views, streams), -8.0)
    for l in range(n_layer):
        res[l].fill_diagonal_(0.0)
        pre[l, :, l % streams] = 0.0
        post[l, :, l % streams] = 0.0
    return {"mhc_res": res, "mhc_pre": pre, "mhc_post": post}


def layer_split(R: torch.Tensor, res_logits, pre_logits, tau: float, iters: int):
    """Returns (branch input [B, T, D], mixed residual streams)."""
    h_res = sinkhorn(res_logits, tau, iters)
    h_pre = torch.softmax(pre_logits, dim=-1)  # [V, S]
    branch_in = mix(R, h_pre.t())[:, 0]
    return branch_in, mix(R, h_res)


def layer_merge(R_mixed: torch.Tensor, branch_out: torch.Tensor, post_logits) -> torch.Tensor:
    h_post = torch.softmax(post_logits, dim=-1)  # [V, S]
    return R_mixed + mix(branch_out[:, None], h_post)

"""Context parallelism over the sequence by an exact prefix of the recurrent state.

The reference scales context only through the recurrent state and TBPTT (it has no
ring attention); linearity of the state makes an exact split possible: rank r holds
tokens [r*Tc, (r+1)*Tc). Per layer each rank computes its chunk's attention from a zero
state plus its chunk state ``rho_r = sum_t gamma^(Tc-t) q_t v_t``; the states are
all-gathered (differentiably) and rank r adds the decayed exclusive prefix
``rho_in(r) = sum_{r'<r} gamma^((r-1-r')Tc) rho_{r'}`` as ``gamma^i q_i rho_in(r)``.
Gradients flow back through the all-gather to earlier ranks. RoPE uses global
positions. This module runs the PyTorch path (any device); the loss is the mean over
all ranks' tokens.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.distributed.nn as dnn

from ..models import reference as R


def _attention(rank: int, world: int, decay, group):
    def attn(q, v):
        B, H, Tc, N = q.shape
        c, rho = R.linear_attention_dense(q, v, decay=decay, need_state=True)
        states = dnn.all_gather(rho.contiguous(), group=group)
        # every rank must take part in the all-gather's backward (a collective): tie the
        # states this rank does not need into the graph with weight zero
        c = c + 0.0 * sum(s.sum() for s in states[rank:])
        if rank > 0:
            rho_in = torch.zeros_like(rho)
            for r in range(rank):
                w = states[r]
                if decay is not None:
                    w = w * (decay.view(1, H, 1, 1) ** ((rank - 1 - r) * Tc))
                rho_in = rho_in + w
            init = torch.matmul(q, rho_in)
            if decay is not None:
                i = torch.arange(Tc, device=q.device, dtype=q.dtype)
                init = init * (decay.view(1, H, 1, 1) ** i.view(1, 1, Tc, 1))
            c = c + init
        return c, None
    return attn


def cp_loss(model, tokens: torch.Tensor, targets: torch.Tensor, group=None) -> torch.Tensor:
    """This rank's chunk [B, Tc] of a sequence split over the group; returns the loss
    mean over the whole sequence (all ranks), differentiable."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    cfg = model.cfg
    p = model.param_dict()
    gamma, beta = p["norm_gamma"], p["norm_beta"]
    norm = R.make_norm(cfg.norm_kind, gamma, beta, cfg.norm_eps, p.get("norm_alpha"), p.get("norm_shift"))
    B, Tc = tokens.shape
    v = norm(p["embed"][tokens])
    Nh = cfg.latent_per_head
    freqs = R.rope_freqs(Nh, cfg.rope_theta, device=v.device, dtype=v.dtype) if cfg.rotary_embedding == "rope" else None
    decay = R.decay_vector(cfg.decay_slopes(), device=v.device, dtype=v.dtype) if cfg.uses_decay() else None
    pos = torch.arange(rank * Tc, (rank + 1) * Tc, device=v.device)
    attn = _attention(rank, world, decay, group)
    for _ in range(cfg.n_layer):
        v, _, _ = R.bdh_layer(v, p["encoder"], p["encoder_v"], p["decoder"], gamma, beta, eps=cfg.norm_eps,
                              thr=cfg.thresholds()[0], thr_y=cfg.thresholds()[1], freqs=freqs, positions=pos, decay=decay, norm=norm,
                              attention=attn)
    head = p["embed"].t() if p.get("lm_head") is None else p["lm_head"]
    return R.cross_entropy(v @ head, targets) / world


def cp_step_grads(model, tokens, targets, group=None) -> torch.Tensor:
    """Loss + gradients summed over the group into ``.grad`` (the full-sequence gradient)."""
    loss = cp_loss(model, tokens, targets, group)
    params = list(model.parameters())
    grads = torch.autograd.grad(loss, params, allow_unused=True)
    for prm, g in zip(params, grads):
        if g is None:
            prm.grad.zero_()
        else:
            prm.grad.copy_(g)
    dist.all_reduce(model.store.grad, group=group)
    total = loss.detach().clone()
    dist.all_reduce(total, group=group)
    return total

"""Neuron-dimension (head-aligned) tensor parallelism.

The reference declares ``ParallelismKind::TensorParallelNeuron`` with a head-aligned
partition (burn_dragon_train/src/config/core.rs:46-77,187-206) but rejects it at run
time; here it runs. Rank r of a group of size P owns heads [r*H/P, (r+1)*H/P): its
slices of ``encoder`` / ``encoder_v`` ([H/P, D, Nh]) and the matching rows of
``decoder`` ([N/P, D]). The residual stream, embedding, LM head and LayerNorm are
replicated. Per layer the only cross-rank traffic is the sum of the decoder partial
``yn_r E_r`` ([M, D] fp32) in the forward and of the residual-gradient partials in the
backward; attention is entirely local to a head. Weight gradients of the sharded
projections stay local; the LayerNorm gradient terms of the local heads are summed.
"""

from __future__ import annotations

import copy

import torch
import torch.distributed as dist


def hybrid_layout(world: int, tp: int) -> tuple[list[list[int]], list[list[int]]]:
    """2-D DP x TP layout (the reference's hybrid_2d, validate.rs:1492-1503): tensor-parallel
    groups are consecutive ranks (one NVSwitch node holds them), data-parallel groups
    stride over them. Returns (tp_groups, dp_groups)."""
    if world % tp:
        raise ValueError(f"world {world} not divisible by tensor-parallel size {tp}")
    tp_groups = [list(range(d * tp, (d + 1) * tp)) for d in range(world // tp)]
    dp_groups = [list(range(i, world, tp)) for i in range(tp)]
    return tp_groups, dp_groups


class TensorParallel:
    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def all_reduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)

    def local_config(self, cfg):
        """This rank's model config: H/P heads of the same Nh, ALiBi slopes of its heads."""
        H, P = cfg.n_head, self.world
        if H % P or cfg.mlp_internal_dim_multiplier % P:
            raise ValueError(f"{H} heads / multiplier {cfg.mlp_internal_dim_multiplier} not divisible by TP size {P}")
        local = copy.deepcopy(cfg)
        slopes = cfg.decay_slopes()
        local.n_head = H // P
        local.mlp_internal_dim_multiplier = cfg.mlp_internal_dim_multiplier // P
        local.alibi_slopes = slopes[self.rank * local.n_head:(self.rank + 1) * local.n_head]
        assert local.latent_per_head == cfg.latent_per_head
        return local

    def head_slice(self, cfg) -> slice:
        h = cfg.n_head // self.world
        return slice(self.rank * h, (self.rank + 1) * h)

    def shard_from_full(self, local_model, full_params: dict, cfg) -> None:
        """Copy this rank's slices of a full model's parameters into ``local_model``."""
        hs = self.head_slice(cfg)
        Nh = cfg.latent_per_head
        rows = slice(hs.start * Nh, hs.stop * Nh)
        with torch.no_grad():
            local_model.encoder.copy_(full_params["encoder"][hs])
            local_model.encoder_v.copy_(full_params["encoder_v"][hs])
            local_model.decoder.copy_(full_params["decoder"][rows])
            for n in ("embed", "lm_head", "norm_gamma", "norm_beta"):
                getattr(local_model, n).copy_(full_params[n])
        local_model.store.refresh_shadow()

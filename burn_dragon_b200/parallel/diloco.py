"""DiLoCo local-SGD: K inner AdamW steps per replica, then an outer Nesterov-momentum SGD
step on the averaged pseudo-gradient (burn_dragon_p2p/src/manifests.rs:218,717-732,1508;
docs/random-scaffold-dragon-report.md:228-291). The reference runs it between WAN peers
over libp2p; here the replicas are ranks of a process group (NCCL or gloo), and the
pseudo-gradient can travel in fp16 (the reference's FP16 codec). With a random scaffold
only the mutable tensors (the adapters) exist in the flat store, so only they move.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class DiLoCo:
    def __init__(self, store, inner_steps: int = 8, outer_lr: float = 0.7, momentum: float = 0.9,
                 nesterov: bool = True, codec: str = "fp32", group=None):
        self.store = store
        self.inner_steps = inner_steps
        self.outer_lr, self.momentum, self.nesterov = outer_lr, momentum, nesterov
        self.codec = codec
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.anchor = store.data.detach().clone()  # the last global parameters
        self.buf = torch.zeros_like(self.anchor)
        self.inner = 0

    def after_inner_step(self) -> bool:
        """Call after every inner optimizer step; returns True when an outer step ran."""
        self.inner += 1
        if self.inner < self.inner_steps:
            return False
        self.inner = 0
        self.outer_step()
        return True

    @torch.no_grad()
    def outer_step(self) -> None:
        delta = self.anchor - self.store.data  # pseudo-gradient of this replica
        if self.codec == "fp16":
            delta = delta.half()
        if self.world > 1:
            dist.all_reduce(delta, group=self.group)
        delta = delta.float() / self.world
        self.buf.mul_(self.momentum).add_(delta)
        step = delta + self.momentum * self.buf if self.nesterov else self.buf
        self.anchor.sub_(self.outer_lr * step)
        self.store.data.copy_(self.anchor)
        self.store.refresh_shadow()

"""Fused AdamW over the flat parameter store, plus learning-rate schedules.

AdamW with decoupled weight decay, beta (0.9, 0.999) defaults and optional global
grad-norm clipping or, when no norm is set, element-wise value clipping (burn_dragon_train/src/config/optimizer.rs:6-460). On CUDA one kernel
updates the fp32 master weights, both moments and the bf16 GEMM shadow in a single
pass over the flat buffers; the clipping coefficient stays on the device.
LR schedules mirror burn_dragon_train/src/train/pipeline/schedule.rs:6-392.
"""

from __future__ import annotations

import math

import torch

from .. import _ext


def lr_at(step: int, base_lr: float, schedule: dict | None, max_iters: int) -> float:
    """Constant / cosine(warmup, min) / linear / exponential / step / noam."""
    sched = dict(schedule or {"type": "constant"})
    kind = sched.get("type", "constant")
    warm = int(sched.get("warmup_iters", 0))
    if warm and step < warm:
        return base_lr * (step + 1) / warm
    if kind == "constant":
        return base_lr
    t = max(0, step - warm)
    span = max(1, max_iters - warm)
    min_lr = float(sched.get("min_lr", 0.0))
    if kind == "cosine":
        c = 0.5 * (1.0 + math.cos(math.pi * min(1.0, t / span)))
        return min_lr + (base_lr - min_lr) * c
    if kind == "linear":
        return base_lr + (min_lr - base_lr) * min(1.0, t / span)
    if kind == "exponential":
        return base_lr * float(sched.get("gamma", 0.999)) ** t
    if kind == "step":
        return base_lr * float(sched.get("gamma", 0.1)) ** (t // int(sched.get("step_size", 1000)))
    if kind == "noam":
        d = float(sched.get("model_dim", 256))
        s = step + 1
        return base_lr * d ** -0.5 * min(s ** -0.5, s * max(1, warm) ** -1.5)
    raise ValueError(f"unknown lr schedule {kind!r}")


class FusedAdamW:
    """AdamW over ``ParamStore`` flat buffers (a boolean mask selects trainable elements)."""

    def __init__(self, store, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.1,
                 grad_clip_norm: float | None = None, grad_clip_value: float | None = None):
        self.store = store
        self.clip_value = grad_clip_value if grad_clip_norm is None else None
        self.lr = lr
        self.b1, self.b2 = betas
        self.eps = eps
        self.wd = weight_decay
        self.clip = grad_clip_norm
        self.m = torch.zeros_like(store.data)
        self.v = torch.zeros_like(store.data)
        self.t = 0
        self._scratch = torch.zeros(4, dtype=torch.float32, device=store.data.device)
        # {lr, 1-b1^t, 1-b2^t} on the device, so a captured step reads this step's values
        self._hyper = torch.zeros(4, dtype=torch.float32, device=store.data.device)
        # pageable on purpose: the copy from pageable memory is staged before copy_ returns,
        # so the next step may overwrite this buffer while the GPU still lags behind
        self._hyper_host = torch.zeros(4, dtype=torch.float32)

    def state_dict(self) -> dict:
        return {"m": self.m, "v": self.v, "t": self.t, "lr": self.lr}

    def load_state_dict(self, sd: dict) -> None:
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        self.t = int(sd["t"])

    def grad_norm(self) -> torch.Tensor:
        return self._scratch[1]

    def prepare(self, lr: float | None = None) -> None:
        """Advance the step counter and stage this step's scalars on the device."""
        self.t += 1
        self._lr_now = self.lr if lr is None else lr
        self._hyper_host[0] = self._lr_now
        self._hyper_host[1] = 1.0 - self.b1 ** self.t
        self._hyper_host[2] = 1.0 - self.b2 ** self.t
        if self.store.data.is_cuda:
            self._hyper.copy_(self._hyper_host, non_blocking=True)

    @torch.no_grad()
    def apply(self) -> None:
        """The update itself (device work only on CUDA; safe to capture in a CUDA graph)."""
        s = self.store
        if self.clip_value is not None:  # burn's GradientClipping::Value: clamp every element
            s.grad.clamp_(-self.clip_value, self.clip_value)
        if s.data.is_cuda:
            mod = _ext.load()
            gscale = None
            if self.clip is not None:
                mod.grad_clip_coef(s.grad, self._scratch, float(self.clip))
                gscale = self._scratch[2:3]
            mod.adamw(s.data, s.grad, self.m, self.v, s.shadow, 0.0, self.b1, self.b2, self.eps, self.wd, 1.0, 1.0,
                      gscale, self._hyper)
            return
        lr = self._lr_now
        bc1, bc2 = float(self._hyper_host[1]), float(self._hyper_host[2])
        g = s.grad
        if self.clip is not None:
            norm = g.norm()
            self._scratch[1] = norm
            g = g * torch.clamp(self.clip / (norm + 1e-6), max=1.0)
        self.m.mul_(self.b1).add_(g, alpha=1 - self.b1)
        self.v.mul_(self.b2).addcmul_(g, g, value=1 - self.b2)
        s.data.mul_(1 - lr * self.wd)
        s.data.addcdiv_(self.m / bc1, (self.v / bc2).sqrt_().add_(self.eps), value=-lr)

    @torch.no_grad()
    def step(self, lr: float | None = None) -> None:
        self.prepare(lr)
        self.apply()

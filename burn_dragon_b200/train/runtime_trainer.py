"""Trainer for configurations that enable a layer-loop variant (``DragonRuntime``).

The BDH core weights keep their flat store and the fused AdamW (one kernel over the
whole buffer on CUDA); the optional modules (attention-residual connector, split slow
weights, latent-reasoning heads, ...) are a handful of small tensors updated with
``torch.optim.AdamW``. Gradients come from autograd over the PyTorch layer path; the
data-parallel mean is one all-reduce of the flat core gradient plus one of the
flattened extra gradients. Stateful TBPTT carries ``RuntimeState`` (rho plus the
auxiliary memories), detached at every chunk boundary.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..config import DragonConfig
from ..models import reference as R
from ..models.dragon_runtime import DragonRuntime, RuntimeState
from .optim import FusedAdamW, lr_at


class RuntimeTrainer:
    def __init__(self, cfg: DragonConfig, device, lr=1e-3, weight_decay=0.1, betas=(0.9, 0.999), eps=1e-8,
                 grad_clip_norm=None, seed=1337, lr_schedule=None, max_iters=1000, rollout_mode: str = "fused",
                 grad_clip_value=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.model = DragonRuntime(cfg, device=self.device, seed=seed, rollout_mode=rollout_mode)
        self.core = self.model.core
        self.opt = FusedAdamW(self.core.store, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                              grad_clip_norm=grad_clip_norm, grad_clip_value=grad_clip_value)
        core_ids = {id(p) for p in self.core.parameters()}
        self.extra_params = [p for p in self.model.parameters() if id(p) not in core_ids]
        self.extra_names = [n for n, p in self.model.named_parameters() if id(p) not in core_ids]
        self.extra_opt = torch.optim.AdamW(self.extra_params, lr=lr, betas=betas, eps=eps,
                                           weight_decay=weight_decay) if self.extra_params else None
        self.base_lr = lr
        self.lr_schedule = lr_schedule
        self.max_iters = max_iters
        self.step_idx = 0
        self.world = dist.get_world_size() if dist.is_initialized() else 1

    def _grads(self, loss: torch.Tensor) -> None:
        core = list(self.core.parameters())
        params = core + self.extra_params
        grads = torch.autograd.grad(loss, params, allow_unused=True)
        for p, g in zip(core, grads[:len(core)]):
            if g is None:
                p.grad.zero_()
            else:
                p.grad.copy_(g)
        for p, g in zip(self.extra_params, grads[len(core):]):
            p.grad = torch.zeros_like(p) if g is None else g
        if self.world > 1:
            sum_op = dist.ReduceOp.SUM
            dist.all_reduce(self.core.store.grad, op=sum_op)
            self.core.store.grad.div_(self.world)
            if self.extra_params:
                flat = torch.cat([p.grad.reshape(-1) for p in self.extra_params])
                dist.all_reduce(flat, op=sum_op)
                flat.div_(self.world)
                off = 0
                for p in self.extra_params:
                    n = p.numel()
                    p.grad.copy_(flat[off:off + n].view_as(p))
                    off += n

    def _update(self) -> None:
        lr = lr_at(self.step_idx, self.base_lr, self.lr_schedule, self.max_iters)
        self.opt.prepare(lr)
        self.opt.apply()
        if self.extra_opt is not None:
            for g in self.extra_opt.param_groups:
                g["lr"] = lr
            if self.opt.clip_value is not None:
                for p in self.extra_params:
                    p.grad.clamp_(-self.opt.clip_value, self.opt.clip_value)
            self.extra_opt.step()
        self.step_idx += 1

    def step(self, tokens, targets, mask=None, event_mask=None) -> torch.Tensor:
        tokens = tokens.to(self.device, non_blocking=True)
        targets = targets.to(self.device, non_blocking=True)
        lrt = getattr(self, "latent_training", None)
        if lrt is not None and lrt.active(self.step_idx):
            # the training-side latent-reasoning terms read the final hidden states
            h = self.model.forward_hidden(tokens, event_mask=event_mask)
            loss = R.cross_entropy(self.model.logits_from_hidden(h), targets, mask)
            aux = lrt.loss(self.model, h, tokens, self.step_idx, targets=targets, mask=mask)
            if aux is not None:
                loss = loss + aux
        else:
            loss = self.model.loss(tokens, targets, mask, event_mask=event_mask)
        self._grads(loss)
        self._update()
        if lrt is not None and lrt.teacher is not None:
            lrt.teacher.update(self.model)
        return loss.detach()

    def step_stream(self, tokens, targets, state: RuntimeState) -> torch.Tensor:
        """TBPTT chunk: continues ``state`` (detached first) and advances it."""
        tokens = tokens.to(self.device, non_blocking=True)
        targets = targets.to(self.device, non_blocking=True)
        state.detach()
        loss = self.model.loss(tokens, targets, state=state)
        self._grads(loss)
        state.detach()
        self._update()
        return loss.detach()

    def extra_state(self) -> dict[str, torch.Tensor]:
        """The optional modules' weights and AdamW moments, for ``RunDir.save(extra=...)``."""
        out = {f"param.{n}": p.detach() for n, p in zip(self.extra_names, self.extra_params)}
        if self.extra_opt is not None:
            for n, p in zip(self.extra_names, self.extra_params):
                st = self.extra_opt.state.get(p)
                if st:
                    out[f"exp_avg.{n}"] = st["exp_avg"]
                    out[f"exp_avg_sq.{n}"] = st["exp_avg_sq"]
                    out[f"step.{n}"] = torch.as_tensor(st["step"], dtype=torch.float32).reshape(1)
        return out

    def load_extra_state(self, sd: dict[str, torch.Tensor]) -> None:
        with torch.no_grad():
            for n, p in zip(self.extra_names, self.extra_params):
                p.copy_(sd[f"param.{n}"].to(p.device, p.dtype))
                if self.extra_opt is not None and f"exp_avg.{n}" in sd:
                    self.extra_opt.state[p] = {
                        "exp_avg": sd[f"exp_avg.{n}"].to(p.device).clone(),
                        "exp_avg_sq": sd[f"exp_avg_sq.{n}"].to(p.device).clone(),
                        "step": torch.tensor(float(sd[f"step.{n}"][0])),
                    }

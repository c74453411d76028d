"""Data parallelism: the NVLink peer-memory gradient step and the NCCL baseline.

``NVLinkDDP`` puts the model's flat parameter / gradient / bf16-shadow buffers in
symmetric device memory shared through CUDA IPC, then runs each optimizer step as
barrier -> fused reduce-scatter + AdamW-on-own-shard + all-gather-by-stores -> barrier
(``csrc/comm.cu``). Every rank keeps the full fp32 master and bf16 shadow (the next
forward needs them) but only its shard of the AdamW moments, so optimizer-state memory
and optimizer math are divided by the world size (a partitioned optimizer, the
reference's intended ZeRO-style mode: burn_dragon_train/src/config/core.rs:87-94).

The NCCL path (``Trainer.allreduce_grads`` without a communicator) mirrors the reference's
process-group DDP: gradient mean over ranks, then a full AdamW on every rank.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _ext


class NVLinkDDP:
    """Symmetric-memory communicator for one flat parameter store of ``numel`` elements."""

    FLAG_WORDS = 64

    def __init__(self, numel: int, device: torch.device, group=None):
        if not dist.is_initialized():
            raise RuntimeError("NVLinkDDP needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("NVLinkDDP supports up to 8 ranks on one NVSwitch node")
        self.device = device
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        mod = _ext.load()
        unit = 4 * self.world
        self.numel = -(-numel // unit) * unit
        self.shard = self.numel // self.world
        self.lo = self.rank * self.shard
        self.hi = self.lo + self.shard
        sizes = {"grad": self.numel * 4, "param": self.numel * 4, "shadow": self.numel * 2, "flags": self.FLAG_WORDS * 4}
        self._own = {k: mod.sym_alloc(b, self.dev) for k, b in sizes.items()}
        handles = {k: mod.ipc_handle(p, self.dev) for k, p in self._own.items()}
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, handles, group=group)
        self.ptrs: dict[str, list[int]] = {k: [] for k in sizes}
        self._opened: list[int] = []
        for r in range(self.world):
            for k in sizes:
                if r == self.rank:
                    self.ptrs[k].append(self._own[k])
                else:
                    p = mod.ipc_open(gathered[r][k], self.dev)
                    self._opened.append(p)
                    self.ptrs[k].append(p)
        self.grad = mod.wrap_ptr(self._own["grad"], self.numel, 0, self.dev)
        self.param = mod.wrap_ptr(self._own["param"], self.numel, 0, self.dev)
        self.shadow = mod.wrap_ptr(self._own["shadow"], self.numel, 1, self.dev)
        self.m = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.v = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        dist.barrier(group=group)

    def _args(self):
        return self.ptrs["grad"], self.ptrs["param"], self.ptrs["shadow"], self.ptrs["flags"]

    def barrier(self, phase: int) -> None:
        _ext.load().peer_barrier(*self._args(), self.rank, phase, self.err)

    def step_adamw(self, opt) -> None:
        """Reduce-scatter + AdamW on this rank's shard + all-gather of the new weights.
        ``opt`` supplies the hyper-parameters and the device-resident {lr, bc1, bc2}."""
        mod = _ext.load()
        self.barrier(0)
        mod.reduce_adamw(*self._args(), self.rank, self.lo, self.hi, self.m, self.v, 0.0, opt.b1, opt.b2, opt.eps,
                         opt.wd, 1.0, 1.0, opt._hyper)
        self.barrier(1)

    def allreduce_mean(self, grad: torch.Tensor | None = None) -> None:
        """Gradient mean in place over the symmetric gradient buffer (no optimizer)."""
        mod = _ext.load()
        self.barrier(0)
        mod.reduce_mean(self.ptrs["grad"], self.ptrs["flags"], self.rank, self.lo, self.hi, self.err)
        self.barrier(1)

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"NVLinkDDP: a peer barrier timed out (code {code})")

    def state_dict(self) -> dict:
        return {"m": self.m, "v": self.v, "lo": self.lo, "hi": self.hi}

    def close(self) -> None:
        mod = _ext.load()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            mod.ipc_close(p, self.dev)
        self._opened = []

"""Training driver: one process per GPU, fused BDH step, DDP gradient all-reduce, AdamW.

``Trainer.step(tokens, targets)`` is the public per-step call: it copies the batch to
the device (non-blocking from pinned memory), runs forward + CE + backward (the fused
sm_100a path on CUDA, the PyTorch path on CPU), averages the flat gradient buffer over
the data-parallel group, applies AdamW and returns the loss as a device tensor.

DDP mirrors the reference's process-group data parallelism (WORLD_SIZE / RANK /
LOCAL_RANK, gradient mean over ranks; burn_dragon_language/src/train/schedule.rs:
10348-10457), but the all-reduce is one collective over the single flat gradient
buffer instead of one per parameter tensor.
"""

from __future__ import annotations

import datetime
import os
import warnings

import torch
import torch.distributed as dist

from ..config import DragonConfig
from ..models.bdh import BDH
from .optim import FusedAdamW, lr_at


def init_distributed() -> tuple[int, int, int]:
    """Initialise torch.distributed from the torchrun environment; returns (rank, world, local)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        # a rank that dies or stalls ends the others' next collective with an error after
        # this long instead of hanging them (BDH_PG_TIMEOUT_S, seconds)
        timeout = datetime.timedelta(seconds=float(os.environ.get("BDH_PG_TIMEOUT_S", "600")))
        dist.init_process_group(backend=backend, timeout=timeout)
    return rank, world, local


class Trainer:
    def __init__(self, cfg: DragonConfig, device, lr=1e-3, weight_decay=0.1, betas=(0.9, 0.999), eps=1e-8,
                 grad_clip_norm=None, seed=1337, lr_schedule=None, max_iters=1000, comm=None, grad_clip_value=None,
                 tensor_parallel: bool = False, micro_batches: int = 1, sequence_parallel: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        self.micro_batches = micro_batches
        if sequence_parallel and not tensor_parallel:
            raise ValueError("sequence_parallel shards the residual stream of a tensor-parallel group")
        self.tp = None
        self.dp_group = None
        dp_world = None
        if tensor_parallel:
            from ..parallel.tp import TensorParallel, hybrid_layout

            world_all = dist.get_world_size() if dist.is_initialized() else 1
            tp_size = world_all if tensor_parallel is True else int(tensor_parallel)
            if tp_size < world_all:
                # hybrid 2-D: tensor parallel inside groups of tp_size, data parallel across
                tp_groups, dp_groups = hybrid_layout(world_all, tp_size)
                pg_tp = [dist.new_group(g) for g in tp_groups]
                pg_dp = [dist.new_group(g) for g in dp_groups]
                r = dist.get_rank()
                self.tp = TensorParallel(pg_tp[r // tp_size], sequence_parallel=sequence_parallel)
                self.dp_group = pg_dp[r % tp_size]
                dp_world = world_all // tp_size
            else:
                self.tp = TensorParallel(sequence_parallel=sequence_parallel)
            local = self.tp.local_config(cfg)
            self.model = BDH(local, device=self.device, seed=seed)
            # replicated tensors share the seed; each rank's heads get their own stream
            g = torch.Generator().manual_seed(seed * 1009 + 17 + self.tp.rank)
            with torch.no_grad():
                for n in ("encoder", "encoder_v", "decoder"):
                    p = getattr(self.model, n)
                    p.copy_(torch.randn(p.shape, generator=g) * cfg.init_std)
            self.model.store.refresh_shadow()
            self.model.tp = self.tp
        else:
            self.model = BDH(cfg, device=self.device, seed=seed)
        self.opt = FusedAdamW(self.model.store, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                              grad_clip_norm=grad_clip_norm, grad_clip_value=grad_clip_value)
        self.lr_schedule = lr_schedule
        self.max_iters = max_iters
        self.base_lr = lr
        self.step_idx = 0
        # data-parallel world (tensor parallelism alone replicates the batch)
        if dp_world is not None:
            self.world = dp_world
        else:
            self.world = 1 if self.tp is not None else (dist.get_world_size() if dist.is_initialized() else 1)
        self.fused = self.device.type == "cuda"
        if self.fused:
            from ..models.bdh_fused import fused_unsupported

            why = fused_unsupported(cfg)
            if why is not None:
                # autograd over the PyTorch path (cuBLAS / ATen kernels), same step semantics
                warnings.warn(f"fused BDH kernels do not implement {why}; training through the PyTorch path")
                self.fused = False
        # comm: None / "nccl" (all-reduce + full AdamW on every rank), "nvlink"
        # (symmetric-memory reduce-scatter + sharded AdamW + all-gather by peer loads and
        # stores, parallel.ddp) or "nvls" (the same step through NVLink multicast objects:
        # in-switch reduction and multicast stores)
        self.comm = None
        if comm in ("nvlink", "nvls") and self.world > 1:
            from ..parallel.ddp import NVLinkDDP

            if grad_clip_value is not None:
                raise ValueError("the NVLink DDP step clips by global norm only; use comm='nccl' for "
                                 "element-wise value clipping")
            self._bucket_of, buckets = self._ddp_buckets()
            # the forward reads the fp32 master of every bucket but the three shared
            # projections (their bf16 shadow only): those buckets all-gather fp32 too
            master_b = {len(buckets) - 1} if buckets else None
            self.comm = NVLinkDDP(self.model.store.numel, self.device, group=self.dp_group,
                                  grad_dtype=os.environ.get("BDH_DDP_GRAD_DTYPE", "bf16"), buckets=buckets,
                                  master_buckets=master_b, transport="nvls" if comm == "nvls" else "p2p")
            self.model.attach_buffers(self.comm.param, self.comm.grad, self.comm.shadow)
            # overlap the per-bucket gradient exchange with the rest of the backward
            # (BDH_DDP_OVERLAP=0: one exchange after the backward)
            self.overlap = (os.environ.get("BDH_DDP_OVERLAP", "1") != "0" and self.fused
                            and not self.model.scaffold and micro_batches == 1)
        self._graph = None
        self._graph_shape = None
        self._graph_launches = 0
        if self.comm is None:
            self.overlap = False

    def _ddp_buckets(self):
        """Buckets of the flat store in the order the fused backward finishes them: the
        three shared projections (final after layer 0's dE / dDy / dDx contractions), then
        everything else (final at the end of the backward). One bucket for layouts
        without the three projections (random scaffold)."""
        st = self.model.store
        names = list(st.shapes)
        if names[:3] != ["encoder", "encoder_v", "decoder"]:
            return {}, None
        cuts = [st.offsets["encoder"], st.offsets["encoder_v"], st.offsets["decoder"], st.offsets[names[3]]]
        buckets = [(cuts[i], cuts[i + 1]) for i in range(3)] + [(cuts[3], st.numel)]
        return {"encoder": 0, "encoder_v": 1, "decoder": 2}, buckets

    def _grad_ready(self, name: str) -> None:
        b = self._bucket_of.get(name)
        if b is not None:
            self.comm.bucket_ready(b, precast=self.comm.grad_bf16)

    def _grad16(self) -> dict | None:
        """bf16 views of the symmetric gradient buffer for the three shared projections
        (their final backward GEMMs write the transport copy directly)."""
        if not self.comm.grad_bf16:
            return None
        st = self.model.store
        return {n: self.comm.gsym[st.offsets[n]:st.offsets[n] + st.view(st.grad, n).numel()].view(st.shapes[n])
                for n in self._bucket_of}

    def sync_params(self) -> None:
        """Make the full fp32 master and the optimizer moments current on every rank (the
        NVLink step keeps them sharded). A collective: every data-parallel rank calls it."""
        if self.comm is None:
            return
        self.comm.sync_master()
        self.comm.gather_moments(self.opt.m, self.opt.v)

    def dp_shard(self) -> tuple[list[tuple[int, int]], torch.Tensor, torch.Tensor, torch.Tensor]:
        """This rank's slices of the flat store with the fp32 master and the AdamW moments of
        those slices (concatenated in slice order): the sharded checkpoint record."""
        if self.comm is None:
            n = self.model.store.numel
            return [(0, n)], self.model.store.data, self.opt.m, self.opt.v
        sl = [(b["lo"], b["hi"]) for b in self.comm.buckets if b["hi"] > b["lo"]]
        return sl, self.comm.param, self.comm.m, self.comm.v

    def after_load(self) -> None:
        """After a checkpoint load into the model and the full optimizer moments: hand this
        rank's slices of the moments to the NVLink communicator."""
        if self.comm is None:
            return
        for b in self.comm.buckets:
            lo, hi, mo = b["lo"], b["hi"], b["moff"]
            n = min(hi, self.opt.m.numel()) - lo
            if n > 0:
                self.comm.m[mo:mo + n].copy_(self.opt.m[lo:lo + n])
                self.comm.v[mo:mo + n].copy_(self.opt.v[lo:lo + n])
        self.comm.master_synced = True

    def enable_cuda_graph(self, tokens: torch.Tensor, targets: torch.Tensor, warmup: int = 2) -> None:
        """Capture forward + backward + all-reduce + AdamW of one step into a CUDA graph.

        The graph replays on static input buffers; ``step`` copies each batch into them.
        Shapes are fixed at capture; a different batch shape falls back to eager steps.
        Warm-up steps run (and train) before the capture.
        """
        from .. import _ext

        assert self.fused, "CUDA graphs need the CUDA path"
        self._sx = torch.empty_like(tokens, device=self.device)
        self._sy = torch.empty_like(targets, device=self.device)
        self._sx.copy_(tokens)
        self._sy.copy_(targets)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._eager_device_step(self._sx, self._sy)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        self.opt.prepare(lr_at(self.step_idx, self.base_lr, self.lr_schedule, self.max_iters))
        before = _ext.launch_count()
        with torch.cuda.graph(g):
            self._begin_update()
            self._sloss = self.compute_grads(self._sx, self._sy)
            self._update()
        self._graph_launches = _ext.launch_count() - before
        self.opt.t -= 1  # the capture itself did not update anything
        self._graph = g
        self._graph_shape = (tuple(tokens.shape), tuple(targets.shape))

    def _begin_update(self) -> None:
        """Before the backward (after ``opt.prepare``): open the overlapped exchange."""
        if self.overlap:
            self.comm.begin_step(self.opt)

    def _update(self) -> None:
        """Gradient reduction + optimizer update (device work only; capturable)."""
        if self.comm is not None:
            self.comm.step_adamw(self.opt)
        else:
            self.allreduce_grads()
            self.opt.apply()

    def _eager_device_step(self, tokens, targets, mask=None) -> torch.Tensor:
        self.opt.prepare(lr_at(self.step_idx, self.base_lr, self.lr_schedule, self.max_iters))
        self._begin_update()
        loss = self.compute_grads(tokens, targets, mask)
        self._update()
        self.step_idx += 1
        return loss

    def compute_grads(self, tokens: torch.Tensor, targets: torch.Tensor, mask=None) -> torch.Tensor:
        n = self.micro_batches
        if self.fused and n > 1:
            B = tokens.shape[0]
            assert B % n == 0, "batch must split evenly into micro-batches"
            b = B // n
            total = None
            for i in range(n):
                sl = slice(i * b, (i + 1) * b)
                li = self.model.fused_step(tokens[sl], targets[sl], None if mask is None else mask[sl],
                                           accumulate=i > 0, loss_scale=1.0 / n)
                total = li if total is None else total + li
            return total
        if self.fused:
            return self.model.fused_step(tokens, targets, mask,
                                         grad_ready=self._grad_ready if self.overlap else None,
                                         grad16=self._grad16() if self.overlap else None)
        self.model.zero_grad(set_to_none=False)
        loss = self.model.loss(tokens, targets, mask)
        grads = torch.autograd.grad(loss, [p for p in self.model.parameters()], allow_unused=True)
        for p, g in zip(self.model.parameters(), grads):
            if g is None:
                p.grad.zero_()
            else:
                p.grad.copy_(g)
        return loss.detach()

    def allreduce_grads(self) -> None:
        if self.world == 1 or self.comm is not None:
            return  # the NVLink communicator reduces inside its fused optimizer step
        op = dist.ReduceOp.AVG if dist.get_backend() == "nccl" else dist.ReduceOp.SUM
        dist.all_reduce(self.model.store.grad, op=op, group=self.dp_group)
        if op == dist.ReduceOp.SUM:
            self.model.store.grad.div_(self.world)

    def step_stream(self, tokens: torch.Tensor, targets: torch.Tensor, state) -> torch.Tensor:
        """Stateful TBPTT step: the chunk continues ``state`` (detached) and advances it."""
        tokens = tokens.to(self.device, non_blocking=True)
        targets = targets.to(self.device, non_blocking=True)
        if self.fused:
            loss = self.model.fused_step(tokens, targets, state=state)
        else:
            self.model.zero_grad(set_to_none=False)
            if state.rhos is not None:
                state.rhos = [r.detach() for r in state.rhos]
            loss = self.model.loss(tokens, targets, state=state)
            grads = torch.autograd.grad(loss, list(self.model.parameters()), allow_unused=True)
            for p, g in zip(self.model.parameters(), grads):
                if g is None:
                    p.grad.zero_()
                else:
                    p.grad.copy_(g)
            state.detach_in_place()
            loss = loss.detach()
        self.opt.prepare(lr_at(self.step_idx, self.base_lr, self.lr_schedule, self.max_iters))
        self._update()
        self.step_idx += 1
        return loss

    def step(self, tokens: torch.Tensor, targets: torch.Tensor, mask=None) -> torch.Tensor:
        if (self._graph is not None and mask is None
                and (tuple(tokens.shape), tuple(targets.shape)) == self._graph_shape):
            from .. import _ext

            self._sx.copy_(tokens, non_blocking=True)
            self._sy.copy_(targets, non_blocking=True)
            self.opt.prepare(lr_at(self.step_idx, self.base_lr, self.lr_schedule, self.max_iters))
            self._graph.replay()
            _ext.add_launches(self._graph_launches)
            self.step_idx += 1
            return self._sloss
        tokens = tokens.to(self.device, non_blocking=True)
        targets = targets.to(self.device, non_blocking=True)
        if mask is not None:
            mask = mask.to(self.device, non_blocking=True)
        self.opt.prepare(lr_at(self.step_idx, self.base_lr, self.lr_schedule, self.max_iters))
        self._begin_update()
        loss = self.compute_grads(tokens, targets, mask)
        self._update()
        self.step_idx += 1
        return loss

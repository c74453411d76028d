"""Pipeline parallelism: planner and runner.

Planner (burn_dragon_train/src/train/pipeline/planner/plan.rs:22-413 semantics): the
layers are partitioned contiguously over ``stages * virtual`` chunks (virtual chunk c
lives on rank ``c % stages``); a schedule is an ordered event list per rank of forward
(F) and backward (B) micro-batch events. We derive every schedule from one
list-scheduling simulation over the dependency graph F(mb, c) <- F(mb, c-1),
B(mb, c) <- B(mb, c+1), B(mb, c) <- F(mb, c), with per-kind policies:

* ``gpipe``   all forwards, then all backwards (B in reverse micro-batch order);
* ``1f1b``    at most ``stages - rank`` micro-batches in flight, backward preferred;
* ``interleaved`` 1F1B over virtual chunks (a rank alternates its chunks).

The simulation uses unit costs (F = 1, B = 2) and reports makespan, bubble fraction and
peak in-flight micro-batches per rank (the reference's plan metrics).

Runner: one process per stage; activations [M, D] and their gradients move by
point-to-point send/recv (the reference emulated these with rooted broadcasts,
burn_dragon_language/src/train/schedule.rs:10502-10750). The shared BDH weights live on
every stage; after the schedule the per-stage weight gradients are summed over the
pipeline group (PipelineSharedWeightSyncKind::AllReducePerStep, core.rs:120-125).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist


# ------------------------------------------------------------------ planner
def partition(n_layers: int, n_chunks: int) -> list[tuple[int, int]]:
    """Contiguous, balanced layer ranges for ``n_chunks`` chunks."""
    if n_chunks > n_layers:
        raise ValueError("more pipeline chunks than layers")
    base, extra = divmod(n_layers, n_chunks)
    out, l0 = [], 0
    for c in range(n_chunks):
        l1 = l0 + base + (1 if c < extra else 0)
        out.append((l0, l1))
        l0 = l1
    return out


@dataclass
class Plan:
    stages: int
    micro: int
    virtual: int
    kind: str
    layers: list[tuple[int, int]]
    events: list[list[tuple[str, int, int]]]  # per rank: (kind, micro-batch, chunk)
    makespan: float = 0.0
    bubble: float = 0.0
    peak_inflight: list[int] = field(default_factory=list)

    def chunks_of(self, rank: int) -> list[int]:
        return [c for c in range(self.stages * self.virtual) if c % self.stages == rank]


def plan(n_layers: int, stages: int, micro: int, kind: str = "1f1b", virtual: int = 1,
         f_cost: float = 1.0, b_cost: float = 2.0) -> Plan:
    if kind not in ("gpipe", "1f1b", "interleaved"):
        raise ValueError(f"unknown pipeline schedule {kind!r}")
    if kind != "interleaved":
        virtual = 1
    C = stages * virtual
    layers = partition(n_layers, C)
    done_f: dict[tuple[int, int], float] = {}
    done_b: dict[tuple[int, int], float] = {}
    free_at = [0.0] * stages
    events: list[list[tuple[str, int, int]]] = [[] for _ in range(stages)]
    inflight = [0] * stages
    peak = [0] * stages
    pending_f = [[(mb, c) for mb in range(micro) for c in range(C) if c % stages == r] for r in range(stages)]
    pending_b = [[(mb, c) for mb in range(micro) for c in range(C) if c % stages == r] for r in range(stages)]
    limit = [stages - r if kind != "gpipe" else micro * virtual for r in range(stages)]
    if kind == "interleaved":
        limit = [virtual * (stages - r) + (virtual - 1) * stages for r in range(stages)]
    total = 2 * micro * C
    t_done = 0
    while t_done < total:
        best = None
        for r in range(stages):
            cands = []
            # ready backwards
            for mb, c in pending_b[r]:
                if (mb, c) not in done_f:
                    continue
                dep = done_b.get((mb, c + 1)) if c + 1 < C else done_f[(mb, c)]
                if c + 1 < C and dep is None:
                    continue
                ready = max(dep, done_f[(mb, c)])
                cands.append(("B", mb, c, ready))
            if kind == "gpipe" and any(pf for pf in pending_f):
                cands = []  # gpipe: no backward until every forward is done
            for mb, c in pending_f[r]:
                if inflight[r] >= limit[r]:
                    break
                dep = done_f.get((mb, c - 1)) if c > 0 else 0.0
                if dep is None:
                    continue
                cands.append(("F", mb, c, dep))
                break  # forwards in order
            if not cands:
                continue
            # policy: earliest start; ties prefer backward (1F1B), then lower micro-batch
            cands.sort(key=lambda e: (max(e[3], free_at[r]), 0 if e[0] == "B" else 1, e[1]))
            kind_e, mb, c, ready = cands[0]
            start = max(ready, free_at[r])
            if best is None or start < best[0]:
                best = (start, r, kind_e, mb, c)
        if best is None:
            raise RuntimeError("pipeline schedule deadlocked")
        start, r, kind_e, mb, c = best
        cost = f_cost if kind_e == "F" else b_cost
        end = start + cost
        free_at[r] = end
        events[r].append((kind_e, mb, c))
        if kind_e == "F":
            done_f[(mb, c)] = end
            pending_f[r].remove((mb, c))
            inflight[r] += 1
            peak[r] = max(peak[r], inflight[r])
        else:
            done_b[(mb, c)] = end
            pending_b[r].remove((mb, c))
            inflight[r] -= 1
        t_done += 1
    makespan = max(free_at)
    busy = micro * C * (f_cost + b_cost)
    p = Plan(stages, micro, virtual, kind, layers, events, makespan, 1.0 - busy / (stages * makespan), peak)
    return p


# ------------------------------------------------------------------ stage computes
class ReferenceStage:
    """PyTorch-path stage (CPU or GPU): autograd through this stage's layers."""

    def __init__(self, model, layer_range: tuple[int, int], first: bool, last: bool):
        from ..models import reference as R

        self.R = R
        self.model = model
        self.l0, self.l1 = layer_range
        self.first, self.last = first, last
        self.saved: dict[int, tuple] = {}

    def forward(self, mb: int, tokens, targets, v_in, scale: float):
        R, cfg = self.R, self.model.cfg
        params = self.model.param_dict()
        gamma, beta = params["norm_gamma"], params["norm_beta"]
        if self.first:
            v = R.layer_norm(params["embed"][tokens], gamma, beta, cfg.norm_eps)
            leaf = None
        else:
            leaf = v_in.detach().requires_grad_(True)
            v = leaf
        T = v.shape[1]
        Nh = cfg.latent_per_head
        freqs = R.rope_freqs(Nh, cfg.rope_theta, dtype=v.dtype) if cfg.rotary_embedding == "rope" else None
        decay = R.decay_vector(cfg.decay_slopes(), dtype=v.dtype) if cfg.uses_decay() else None
        pos = torch.arange(T)
        for _ in range(self.l0, self.l1):
            v, _, _ = R.bdh_layer(v, params["encoder"], params["encoder_v"], params["decoder"], gamma, beta,
                                  eps=cfg.norm_eps, thr=cfg.thresholds()[0], thr_y=cfg.thresholds()[1], freqs=freqs, positions=pos, decay=decay)
        loss = None
        if self.last:
            head = params["embed"].t() if params.get("lm_head") is None else params["lm_head"]
            loss = R.cross_entropy(v @ head, targets) * scale
        self.saved[mb] = (leaf, v, loss)
        return v.detach(), (loss.detach() if loss is not None else None)

    def backward(self, mb: int, dv_out):
        leaf, v, loss = self.saved.pop(mb)
        params = [p for p in self.model.parameters()]
        if self.last:
            outs = torch.autograd.grad(loss, params + ([leaf] if leaf is not None else []), allow_unused=True)
        else:
            outs = torch.autograd.grad(v, params + ([leaf] if leaf is not None else []), grad_outputs=dv_out,
                                       allow_unused=True)
        for p, g in zip(params, outs[:len(params)]):
            if g is not None:
                p.grad.add_(g)
        return outs[len(params)] if leaf is not None else None


class FusedStage:
    """sm_100a stage: one fused workspace per micro-batch slot."""

    def __init__(self, model, layer_range: tuple[int, int], first: bool, last: bool, batch: int, seq: int):
        import copy

        from ..models.bdh_fused import FusedBDH, FusedWorkspace

        self.model = model
        self.first, self.last = first, last
        cfg = copy.deepcopy(model.cfg)
        cfg.n_layer = layer_range[1] - layer_range[0]
        self.cfg = cfg
        self.pool: list = []
        self.free: list = []
        self.slot: dict[int, object] = {}
        self._make = lambda: FusedBDH(cfg, FusedWorkspace(cfg, batch, seq, model.store.data.device))  # noqa: E731
        self.first_backward = True

    def _get(self):
        if self.free:
            return self.free.pop()
        f = self._make()
        self.pool.append(f)
        return f

    def forward(self, mb: int, tokens, targets, v_in, scale: float):
        f = self._get()
        self.slot[mb] = f
        p32 = self.model.store.views(self.model.store.data)
        p16 = self.model.shadow_dict()
        f.forward(p16, p32, tokens, v_in=None if self.first else v_in, with_head=self.last)
        loss = f.loss(targets, scale=scale) if self.last else None
        return f.ws.v32[f.ws.L], loss

    def backward(self, mb: int, dv_out):
        f = self.slot.pop(mb)
        p32 = self.model.store.views(self.model.store.data)
        p16 = self.model.shadow_dict()
        dv = f.backward(p16, p32, self.model.grad_dict(), self._tokens.pop(mb, None), pos0=0,
                        accumulate=not self.first_backward, dv_out=None if self.last else dv_out,
                        with_embed=self.first)
        self.first_backward = False
        self.free.append(f)
        return dv


# ------------------------------------------------------------------ runner
class PipelineRunner:
    """Executes one rank's event list for a step (virtual = 1 at run time)."""

    def __init__(self, model, plan_: Plan, rank: int, batch: int, seq: int, group=None, fused: bool | None = None):
        if plan_.virtual != 1:
            raise ValueError("the runner executes one chunk per rank (interleaved plans are simulated only)")
        self.model, self.plan, self.rank, self.group = model, plan_, rank, group
        self.first = rank == 0
        self.last = rank == plan_.stages - 1
        rng = plan_.layers[rank]
        fused = model.store.data.is_cuda if fused is None else fused
        if fused:
            self.stage = FusedStage(model, rng, self.first, self.last, batch, seq)
            self.stage._tokens = {}
        else:
            self.stage = ReferenceStage(model, rng, self.first, self.last)
        self.D = model.cfg.n_embd
        self.ranks = [dist.get_global_rank(group, r) if group is not None else r for r in range(plan_.stages)]

    def step(self, tokens: torch.Tensor, targets: torch.Tensor) -> torch.Tensor | None:
        """Run all micro-batches of one step; grads end summed over the pipeline group.
        Returns the mean loss on the last stage (None elsewhere)."""
        m = self.plan.micro
        B = tokens.shape[0]
        b = B // m
        dev = self.model.store.data.device
        T = tokens.shape[1]
        if isinstance(self.stage, FusedStage):
            self.stage.first_backward = True
        else:
            self.model.store.grad.zero_()
        losses = []
        sends = []
        events = self.plan.events[self.rank]
        pending: dict[int, tuple] = {}

        def post_recv(k: int) -> None:
            # The activation (F) or gradient (B) this event consumes, received without
            # blocking the host: the wait is a stream dependency, so the host keeps
            # enqueueing and the transfer overlaps the compute already queued. Posted only
            # after the previous event's send, which keeps every rank pair's NCCL
            # operations in the same order on both sides.
            if k >= len(events) or k in pending:
                return
            kind = events[k][0]
            if kind == "F" and not self.first:
                buf = torch.empty(b, T, self.D, device=dev)
                pending[k] = (dist.irecv(buf, src=self.ranks[self.rank - 1], group=self.group), buf)
            elif kind != "F" and not self.last:
                buf = torch.empty(b, T, self.D, device=dev)
                pending[k] = (dist.irecv(buf, src=self.ranks[self.rank + 1], group=self.group), buf)

        post_recv(0)
        for k, (kind, mb, _) in enumerate(events):
            sl = slice(mb * b, (mb + 1) * b)
            got = None
            if k in pending:
                work, got = pending.pop(k)
                work.wait()
            if kind == "F":
                if isinstance(self.stage, FusedStage):
                    self.stage._tokens[mb] = tokens[sl]
                v_out, loss = self.stage.forward(mb, tokens[sl], targets[sl], got, 1.0 / m)
                if loss is not None:
                    losses.append(loss)
                if not self.last:
                    buf = v_out.reshape(b, T, self.D).clone()  # the workspace slot is reused
                    sends.append((dist.isend(buf, dst=self.ranks[self.rank + 1], group=self.group), buf))
            else:
                dv_in = self.stage.backward(mb, got)
                if not self.first:
                    buf = dv_in.reshape(b, T, self.D).clone()
                    sends.append((dist.isend(buf, dst=self.ranks[self.rank - 1], group=self.group), buf))
            post_recv(k + 1)
        for h, _ in sends:
            h.wait()
        dist.all_reduce(self.model.store.grad, group=self.group)
        return torch.stack(losses).sum() if losses else None

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


class PeerSum:
    """The per-layer decoder sum of tensor parallelism over NVLink peer memory.

    Backward: the residual-gradient partials are summed the same way (``all_reduce_rows``:
    row scatter by P2P stores, owner sums, all-gather by P2P stores).

    The decoder GEMM of every rank stores each output row straight into the slot of the
    rank that owns that row (``EPI_F32_SCATTER``: the reduce-scatter happens in the
    GEMM epilogue, tile by tile, while the tensor cores keep running); after a peer
    barrier each owner sums its W slots and stores the total rows into every rank's
    per-layer sum buffer (``tp_reduce_gather``, an all-gather by P2P stores), and a
    second barrier publishes them. The slot and sum buffers live in symmetric device
    memory shared through CUDA IPC, like the data-parallel communicator's.
    """

    FLAG_WORDS = 64

    def __init__(self, tp: "TensorParallel", M: int, D: int, L: int, device: torch.device):
        from .. import _ext

        W = tp.world
        sp = tp.sequence_parallel
        if M % W:
            raise ValueError(f"token rows {M} must split evenly over {W} tensor-parallel ranks")
        mod = _ext.load()
        self.tp, self.M, self.D, self.L = tp, M, D, L
        self.rows = M // W
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        sizes = {"slots": W * self.rows * D * 4, "sum": (0 if sp else L) * M * D * 4 + 16, "bsum": M * D * 4,
                 "flags": self.FLAG_WORDS * 4}
        if sp:
            # sequence parallel: the bf16 residual operand of every layer and the bf16 decoder
            # gradient are gathered by rows; the fp32 sums stay with their owner
            sizes["v16"] = (L + 1) * M * D * 2
            sizes["dm16"] = M * D * 2
        self._own = {k: mod.sym_alloc(b, self.dev) for k, b in sizes.items()}
        handles = {k: mod.ipc_handle(v, self.dev) for k, v in self._own.items()}
        gathered: list = [None] * W
        dist.all_gather_object(gathered, handles, group=tp.group)
        self.ptrs: dict[str, list[int]] = {k: [] for k in sizes}
        self._opened: list[int] = []
        for r in range(W):
            for k in sizes:
                if r == tp.rank:
                    self.ptrs[k].append(self._own[k])
                else:
                    h = mod.ipc_open(gathered[r][k], self.dev)
                    self._opened.append(h)
                    self.ptrs[k].append(h)
        self.slots = mod.wrap_ptr(self._own["slots"], W * self.rows * D, 0, self.dev)
        if sp:
            self.sum_views = None
            v16 = mod.wrap_ptr(self._own["v16"], (L + 1) * M * D, 1, self.dev).view(L + 1, M, D)
            self.v16_views = [v16[l] for l in range(L + 1)]
            self.dm16 = mod.wrap_ptr(self._own["dm16"], M * D, 1, self.dev).view(M, D)
            self.m_own = torch.empty(L, self.rows, D, device=device)
        else:
            sums = mod.wrap_ptr(self._own["sum"], L * M * D, 0, self.dev).view(L, M, D)
            self.sum_views = [sums[l] for l in range(L)]
        self.bsum = mod.wrap_ptr(self._own["bsum"], M * D, 0, self.dev).view(M, D)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        dist.barrier(group=tp.group)

    def scatter_args(self) -> list[int]:
        W = self.tp.world
        return [W, self.rows, self.tp.rank, self.rows * self.D] + list(self.ptrs["slots"])

    def _barrier(self, phase: int) -> None:
        from .. import _ext

        f = self.ptrs["flags"]
        _ext.load().peer_barrier(f, f, f, f, self.tp.rank, phase, self.err)

    def finish(self, layer: int) -> None:
        """After the scattered GEMM: sum this rank's rows, all-gather them into every
        rank's sum buffer of ``layer``."""
        from .. import _ext

        self._barrier(0)
        base = self.ptrs["sum"]
        dst = [b + layer * self.M * self.D * 4 for b in base]
        _ext.load().tp_reduce_gather(self.slots, dst, self.tp.rank, self.rows, self.M, self.D, self.rows * self.D)
        self._barrier(1)

    def all_reduce_rows(self, t: torch.Tensor) -> None:
        """In-place sum over the group of a local fp32 [M, D] tensor (the backward's
        residual-gradient partials): rows scattered to their owners by P2P stores, owners
        sum and all-gather into the symmetric ``bsum`` buffer, then copied back."""
        from .. import _ext

        mod = _ext.load()
        mod.tp_scatter_rows(t, self.ptrs["slots"], self.tp.rank, self.rows, self.M, self.D, self.rows * self.D)
        self._barrier(0)
        mod.tp_reduce_gather(self.slots, self.ptrs["bsum"], self.tp.rank, self.rows, self.M, self.D,
                             self.rows * self.D)
        self._barrier(1)
        t.view(self.M, self.D).copy_(self.bsum)

    # ---- sequence parallel (``TensorParallel(sequence_parallel=True)``)
    def own_rows(self) -> slice:
        r0 = self.tp.rank * self.rows
        return slice(r0, r0 + self.rows)

    def sp_tail_forward(self, layer: int, v32_in, v32_out, tst, gamma, beta, eps: float, nk: dict | None = None) -> None:
        """After the scattered decoder GEMM of ``layer``: the owner sums its rows' partials,
        runs the residual merge v' = LN(v + LN(m)) on its rows only, and all-gathers the
        bf16 rows of v' (the next GEMM operand) by P2P stores. The fp32 residual stays
        with its owner."""
        from .. import _ext

        mod = _ext.load()
        W, D, rows = self.tp.world, self.D, self.rows
        own = self.own_rows()
        self._barrier(0)
        mod.tp_sum_slots(self.slots, self.m_own[layer], W, rows * D, rows * D, None)
        v16 = self.v16_views[layer + 1]
        mod.tail_fwd(self.m_own[layer], 1, rows * D, v32_in[own], rows, D, gamma, beta, eps, None, v32_out[own],
                     v16[own], tst[own], **(nk or {}))
        self._gather16(self.ptrs["v16"], (layer + 1) * self.M * D * 2 + own.start * D * 2, rows * D * 2)
        self._barrier(1)

    def _gather16(self, ptrs, offset: int, nbytes: int) -> None:
        from .. import _ext

        _ext.load().tp_gather_bytes(ptrs, self.tp.rank, offset, nbytes, self.dev)

    def sp_gather_dm(self) -> None:
        """All-gather this rank's rows of the bf16 decoder gradient (written into ``dm16``)."""
        own = self.own_rows()
        self._barrier(0)  # every rank has finished reading the previous layer's dm16
        self._gather16(self.ptrs["dm16"], own.start * self.D * 2, self.rows * self.D * 2)
        self._barrier(1)

    def sp_reduce_scatter(self, t: torch.Tensor, add_own: torch.Tensor | None = None) -> None:
        """Sum a local fp32 [M, D] partial over the group into this rank's rows of ``t``
        only (rows scattered to their owners by P2P stores, the owner adds its slots and
        ``add_own``); the other rows of ``t`` are left stale."""
        from .. import _ext

        mod = _ext.load()
        W, D, rows, M = self.tp.world, self.D, self.rows, self.M
        own = self.own_rows()
        self._barrier(0)  # every owner has consumed the previous contents of its slots
        mod.tp_scatter_rows(t, self.ptrs["slots"], self.tp.rank, rows, M, D, rows * D)
        self._barrier(1)
        mod.tp_sum_slots(self.slots, t.view(M, D)[own], W, rows * D, rows * D, add_own)

    def check(self) -> None:
        if int(self.err.item()):
            raise RuntimeError(f"tensor-parallel peer barrier timed out (code {int(self.err.item())})")


class TensorParallel:
    def __init__(self, group=None, fused_comm: bool | None = None, sequence_parallel: bool = False):
        """``fused_comm``: run the forward decoder sums through ``PeerSum`` (default on
        CUDA unless BDH_TP_FUSED=0); otherwise NCCL all-reduce.

        ``sequence_parallel``: the residual stream between the tensor-parallel regions is
        sharded by token rows (the reference's ``parallel.tensor.sequence_parallel``):
        each rank owns M / P rows of the fp32 residual, runs the residual merge, the
        LayerNorm backward of the merge and the embedding on those rows only, and the
        ranks exchange bf16 rows (the GEMM operands) instead of fp32 sums. Needs the
        peer-memory path and M divisible by P."""
        import os

        self.group = group
        self.sequence_parallel = sequence_parallel
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if fused_comm is None:
            fused_comm = os.environ.get("BDH_TP_FUSED", "1") != "0" and torch.cuda.is_available()
        self.fused_comm = fused_comm and self.world > 1
        self.peer: PeerSum | None = None

    def attach_peer(self, M: int, D: int, L: int, device: torch.device) -> PeerSum | None:
        """Symmetric buffers for a workspace shape (re-created when the shape changes)."""
        if not self.fused_comm:
            return None
        if self.sequence_parallel and not self.fused_comm:
            raise ValueError("sequence_parallel runs on the peer-memory tensor-parallel path (BDH_TP_FUSED=1, CUDA)")
        p = self.peer
        if p is None or (p.M, p.D, p.L) != (M, D, L):
            self.peer = PeerSum(self, M, D, L, device)
        return self.peer

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

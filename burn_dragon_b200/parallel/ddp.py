"""Data parallelism: the NVLink peer-memory optimizer step and the NCCL baseline.

``NVLinkDDP`` shares, through CUDA IPC, one symmetric region per rank holding the bf16
gradient buffer (or fp32 with ``grad_dtype="fp32"``), the bf16 weight shadow the GEMMs
read, and a page of flags. Each optimizer step is

    cast fp32 grads -> bf16 (local) -> barrier -> ddp_step -> barrier

per bucket of the flat store (``buckets``), each on a side stream as soon as the
backward has finished that bucket's gradients (``overlap``), then a closing barrier

where ``ddp_step`` (``csrc/comm.cu``) is one kernel: rank r sums its slice [lo_r, hi_r)
of every peer's gradient with plain P2P loads (a reduce-scatter, fp32 accumulation),
runs AdamW on its fp32 master slice and moment shard, and stores the new bf16 weights
into every peer's shadow (an all-gather by P2P stores). For the buckets whose fp32 master
the model reads (the embedding, norms and scaffold adapters: ``master_buckets``) the new
fp32 values are stored into every peer as well. For the shared projections a rank keeps
the fp32 master current only on its own slice (ZeRO-1 style: optimizer state and master updates are
partitioned, the reference's intended FSDP mode, burn_dragon_train/src/config/core.rs:
87-94); ``sync_master()`` all-gathers the full fp32 master when a caller needs it
(checkpoints, the PyTorch path, evaluation in fp32).

Global-norm clipping: the peer sum runs first into a local fp32 shard while summing its
squares, the ranks exchange those sums over the flag page (``ddp_norm_exchange``), and
the update applies the common clip coefficient (``ddp_apply``).

Bytes over NVLink per rank and step: (W-1)/W * P * 2 in and out (P parameters, bf16),
against (W-1)/W * P * 4 in and * 6 out for an fp32-gradient, fp32-master step.

The NCCL path (``Trainer.allreduce_grads`` without a communicator) mirrors the reference's
process-group DDP: gradient mean over ranks, then a full AdamW on every rank
(burn_dragon_language/src/train/schedule.rs:10348-10457).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _ext


class NVLinkDDP:
    """Symmetric-memory communicator for one flat parameter store of ``numel`` elements.

    ``buckets``: contiguous [start, end) ranges of the flat store that become final at
    different points of the backward (default: one bucket). Every rank owns an 8-aligned
    1/W slice of every bucket. With ``overlap`` the backward calls ``bucket_ready(b)`` as
    soon as bucket b's gradients are final, and that bucket's cast, barrier and fused
    reduce-scatter + AdamW + all-gather run on a side stream beside the rest of the
    backward; ``step_adamw`` then launches what is left and joins."""

    FLAG_WORDS = 512

    def __init__(self, numel: int, device: torch.device, group=None, grad_dtype: str = "bf16",
                 buckets: list[tuple[int, int]] | None = None, master_buckets: set[int] | None = None,
                 transport: str = "p2p"):
        """``master_buckets``: buckets whose fp32 master the model reads in its forward /
        backward (embedding, norms, scaffold adapters); their new fp32 values are
        all-gathered with the shadow. Default: every bucket.

        ``transport``: "p2p" (CUDA-IPC buffers; the owner loads every peer's gradient and
        stores into every peer's shadow) or "nvls" (the buffers come from torch's symmetric
        memory with one NVLink multicast object each: the owner's gradient sum is one
        ``multimem.ld_reduce`` reduced inside the NVSwitch, its new weights one
        ``multimem.st`` delivered to every rank). The barriers use plain peer stores in
        both."""
        if not dist.is_initialized():
            raise RuntimeError("NVLinkDDP needs an initialised process group")
        if grad_dtype not in ("bf16", "fp32"):
            raise ValueError("grad_dtype must be 'bf16' or 'fp32'")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("NVLinkDDP supports up to 8 ranks on one NVSwitch node")
        self.device = device
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        self.grad_bf16 = grad_dtype == "bf16"
        mod = _ext.load()
        self.numel = -(-numel // 64) * 64
        buckets = buckets or [(0, self.numel)]
        if buckets[0][0] != 0 or buckets[-1][1] < numel or any(a[1] != b[0] for a, b in zip(buckets, buckets[1:])):
            raise ValueError("buckets must tile [0, numel) in order")
        buckets = [(a, b) for a, b in buckets[:-1]] + [(buckets[-1][0], self.numel)]
        if any(a % 8 for a, _ in buckets) or len(buckets) > 50:
            raise ValueError("bucket starts must be multiples of 8 (at most 50 buckets)")
        # every rank's slice of every bucket: [lo, hi), 8-aligned, the last one clipped
        self.buckets = []
        moff = 0
        for a, b in buckets:
            c = -(-(b - a) // (8 * self.world)) * 8
            lo = min(a + self.rank * c, b)
            hi = min(lo + c, b)
            self.buckets.append({"start": a, "end": b, "lo": lo, "hi": hi, "moff": moff})
            moff += hi - lo
        self.shard_total = moff
        # kept for callers of the one-bucket layout
        self.lo, self.hi = self.buckets[0]["lo"], self.buckets[0]["hi"]
        self.shard = -(-self.numel // self.world)
        gbytes = self.numel * (2 if self.grad_bf16 else 4)
        sizes = {"gsym": gbytes, "shadow": self.numel * 2, "flags": self.FLAG_WORDS * 4, "param": self.numel * 4}
        if transport not in ("p2p", "nvls"):
            raise ValueError("transport must be 'p2p' or 'nvls'")
        self.transport = transport
        self.ptrs: dict[str, list[int]] = {k: [] for k in sizes}
        self._opened: list[int] = []
        self.mc: dict[str, int] = {}
        self._symm: dict = {}
        if transport == "nvls":
            self._own = self._nvls_alloc(sizes, group)
        else:
            self._own = {k: mod.sym_alloc(b, self.dev) for k, b in sizes.items()}
            handles = {k: mod.ipc_handle(p, self.dev) for k, p in self._own.items()}
            gathered: list = [None] * self.world
            dist.all_gather_object(gathered, handles, group=group)
            for r in range(self.world):
                for k in sizes:
                    if r == self.rank:
                        self.ptrs[k].append(self._own[k])
                    else:
                        p = mod.ipc_open(gathered[r][k], self.dev)
                        self._opened.append(p)
                        self.ptrs[k].append(p)
        # local fp32 gradient (written by the backward) and fp32 master (current on the
        # owned slices)
        self.grad = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.param = mod.wrap_ptr(self._own["param"], self.numel, 0, self.dev)
        self.master_buckets = set(range(len(self.buckets))) if master_buckets is None else set(master_buckets)
        self.shadow = mod.wrap_ptr(self._own["shadow"], self.numel, 1, self.dev)
        self.gsym = mod.wrap_ptr(self._own["gsym"], self.numel, 1 if self.grad_bf16 else 0, self.dev)
        self.flags_local = mod.wrap_ptr(self._own["flags"], self.FLAG_WORDS, 2, self.dev)
        self.m = torch.zeros(max(1, moff), dtype=torch.float32, device=device)
        self.v = torch.zeros(max(1, moff), dtype=torch.float32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self._gred = None
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=device)
        self.norm_out = torch.zeros(2, dtype=torch.float32, device=device)  # {clip coef, grad norm}
        self.master_synced = True
        self.side = torch.cuda.Stream(device)
        self._launched: set[int] = set()
        self._opt = None
        dist.barrier(group=group)

    def _nvls_alloc(self, sizes: dict, group) -> dict:
        """Allocate every region from torch's symmetric memory and rendezvous it across the
        group: the peers' addresses fill ``ptrs``, the multicast address ``mc``. Raises when
        the system has no multicast support (no NVSwitch multicast objects)."""
        import torch.distributed._symmetric_memory as symm

        grp = group if group is not None else dist.group.WORLD
        if hasattr(symm, "enable_symm_mem_for_group"):
            try:
                symm.enable_symm_mem_for_group(grp.group_name)
            except Exception:  # noqa: BLE001 - newer releases enable every group
                pass
        own = {}
        for k, nbytes in sizes.items():
            t = symm.empty(-(-nbytes // 16) * 16, dtype=torch.uint8, device=self.device)
            t.zero_()
            h = symm.rendezvous(t, grp)
            if k != "flags":
                mc = int(h.multicast_ptr)  # 0 where the device / driver has no multicast support
                if mc == 0:
                    raise RuntimeError("transport='nvls' needs NVLink multicast (NVSwitch) support on every rank")
                self.mc[k] = mc
            self._symm[k] = (t, h)
            self.ptrs[k] = [int(x) for x in h.buffer_ptrs]
            own[k] = int(t.data_ptr())
        torch.cuda.synchronize(self.device)
        return own

    # ---------------------------------------------------------------- per-step protocol
    def begin_step(self, opt) -> None:
        """Start a step on the current stream: advance the step epoch. ``opt`` supplies
        the hyper-parameters (its device scalars must be staged for this step)."""
        _ext.load().ddp_epoch_advance(self.flags_local)
        self._launched = set()
        self._opt = opt
        if opt.clip is not None and self._gred is None:
            self._gred = torch.empty(max(1, self.shard_total), dtype=torch.float32, device=self.device)
        if opt.clip is not None:
            self._sumsq.zero_()

    def _bucket_work(self, b: int, precast: bool = False) -> None:
        mod = _ext.load()
        bk = self.buckets[b]
        a, e, lo, hi = bk["start"], bk["end"], bk["lo"], bk["hi"]
        opt = self._opt
        if precast:
            pass  # the backward wrote this bucket's transport copy itself
        elif self.grad_bf16:
            mod.cast_bf16(self.grad[a:e], self.gsym[a:e])
        else:
            self.gsym[a:e].copy_(self.grad[a:e])
        mod.ddp_slot_barrier(self.ptrs["flags"], self.rank, b, self.err)
        if hi <= lo:
            return
        g, sh = self.ptrs["gsym"], self.ptrs["shadow"]
        mo, n = bk["moff"], hi - lo
        gm = self.ptrs["param"] if b in self.master_buckets else []
        if self.transport == "nvls":
            mcm = self.mc["param"] if b in self.master_buckets else 0
            if opt.clip is None:
                mod.ddp_step_nvls(self.mc["gsym"], self.mc["shadow"], mcm, self.grad_bf16, self.world, lo, hi,
                                  self.param, self.m[mo:mo + n], self.v[mo:mo + n], opt.b1, opt.b2, opt.eps, opt.wd,
                                  opt._hyper, None)
            else:
                part = self._bucket_sumsq(b)
                mod.ddp_reduce_nvls(self.mc["gsym"], self.grad_bf16, self.world, lo, hi, self._gred[mo:mo + n], part)
                self._sumsq.add_(part)
            return
        if opt.clip is None:
            mod.ddp_step(g, sh, self.grad_bf16, self.rank, lo, hi, self.param, self.m[mo:mo + n], self.v[mo:mo + n],
                         opt.b1, opt.b2, opt.eps, opt.wd, opt._hyper, None, gm)
        else:
            # sums of squares accumulate into _sumsq over the buckets (ddp_reduce zeroes its
            # target, so each bucket reduces into a scratch word first)
            part = self._bucket_sumsq(b)
            mod.ddp_reduce(g, sh, self.grad_bf16, self.rank, lo, hi, self._gred[mo:mo + n], part)
            self._sumsq.add_(part)

    def _bucket_sumsq(self, b: int) -> torch.Tensor:
        if not hasattr(self, "_bsum"):
            self._bsum = torch.zeros(len(self.buckets), dtype=torch.float32, device=self.device)
        return self._bsum[b:b + 1]

    def bucket_ready(self, b: int, precast: bool = False) -> None:
        """Bucket b's gradients are final on the current stream and this rank no longer
        reads its shadow weights before the step ends: run its communication on the side
        stream from here on. ``precast``: the bucket's transport copy (bf16) is already in
        the symmetric gradient buffer."""
        if b in self._launched:
            return
        self._launched.add(b)
        cur = torch.cuda.current_stream(self.device)
        self.side.wait_stream(cur)
        with torch.cuda.stream(self.side):
            self._bucket_work(b, precast)

    def step_adamw(self, opt) -> None:
        """Finish the step: launch the buckets not yet launched, join the side stream, and
        (with global-norm clipping) exchange the norm and apply the clipped update; then
        the closing barrier after which every rank's shadow holds the new weights."""
        mod = _ext.load()
        if self._opt is None:
            self.begin_step(opt)
        for b in range(len(self.buckets)):
            self.bucket_ready(b)
        cur = torch.cuda.current_stream(self.device)
        cur.wait_stream(self.side)
        if opt.clip is not None:
            mod.ddp_norm_exchange(self.ptrs["flags"], self.rank, self._sumsq, float(opt.clip), self.norm_out, self.err)
            g, sh = self.ptrs["gsym"], self.ptrs["shadow"]
            for b, bk in enumerate(self.buckets):
                lo, hi, mo = bk["lo"], bk["hi"], bk["moff"]
                if hi > lo and self.transport == "nvls":
                    n = hi - lo
                    mcm = self.mc["param"] if b in self.master_buckets else 0
                    mod.ddp_apply_nvls(self.mc["shadow"], mcm, lo, hi, self._gred[mo:mo + n], self.param,
                                       self.m[mo:mo + n], self.v[mo:mo + n], opt.b1, opt.b2, opt.eps, opt.wd,
                                       opt._hyper, self.norm_out)
                elif hi > lo:
                    n = hi - lo
                    gm = self.ptrs["param"] if b in self.master_buckets else []
                    mod.ddp_apply(g, sh, self.rank, lo, hi, self._gred[mo:mo + n], self.param, self.m[mo:mo + n],
                                  self.v[mo:mo + n], opt.b1, opt.b2, opt.eps, opt.wd, opt._hyper, self.norm_out, gm)
            opt._scratch[1:2].copy_(self.norm_out[1:2])
        mod.ddp_slot_barrier(self.ptrs["flags"], self.rank, len(self.buckets), self.err)
        self._opt = None
        self.master_synced = False

    def sync_master(self) -> None:
        """All-gather the fp32 master slices so every rank holds the full current master."""
        if self.master_synced:
            return
        if self.world > 1:
            for b, bk in enumerate(self.buckets):
                if b in self.master_buckets:
                    continue  # already current on every rank
                a, e = bk["start"], bk["end"]
                c = -(-(e - a) // (8 * self.world)) * 8
                full = torch.zeros(c * self.world, dtype=torch.float32, device=self.device)
                mine = torch.zeros(c, dtype=torch.float32, device=self.device)
                mine[:bk["hi"] - bk["lo"]].copy_(self.param[bk["lo"]:bk["hi"]])
                dist.all_gather_into_tensor(full, mine, group=self.group)
                self.param[a:e].copy_(full[:e - a])
        self.master_synced = True

    def gather_moments(self, m_full: torch.Tensor, v_full: torch.Tensor) -> None:
        """Assemble the full AdamW moments from every rank's slices (a collective)."""
        for src, dst in ((self.m, m_full), (self.v, v_full)):
            for bk in self.buckets:
                a, e = bk["start"], bk["end"]
                c = -(-(e - a) // (8 * self.world)) * 8
                full = torch.zeros(c * self.world, dtype=torch.float32, device=self.device)
                mine = torch.zeros(c, dtype=torch.float32, device=self.device)
                n = bk["hi"] - bk["lo"]
                mine[:n].copy_(src[bk["moff"]:bk["moff"] + n])
                if self.world > 1:
                    dist.all_gather_into_tensor(full, mine, group=self.group)
                else:
                    full.copy_(mine)
                lim = min(e, dst.numel())
                if lim > a:
                    dst[a:lim].copy_(full[:lim - a])

    def check(self) -> None:
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"NVLinkDDP: a peer wait timed out (code {code})")

    def state_dict(self) -> dict:
        return {"m": self.m, "v": self.v, "buckets": [dict(b) for b in self.buckets]}

    def close(self) -> None:
        mod = _ext.load()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            mod.ipc_close(p, self.dev)
        self._opened = []

"""Metrics sinks and the stage profiler.

* ``MetricsLogger``: one JSON object per logged step in ``<run>/events/metrics.jsonl``
  (loss, lr, grad norm, device-timed step ms, tokens/s) plus rank-0 console lines — the
  JSONL file sink of the reference's event bus (burn_dragon_train/src/train/events.rs,
  metrics.rs:43-625).
* ``StageProfiler``: per-phase device time with CUDA events (host clock on CPU), enabled
  by ``DragonModel_STAGE_PROFILE`` as in the reference (burn_dragon_language/src/train/
  profile.rs:1-576). Its summary reports ``wall_tokens_per_second``,
  ``model_tokens_per_second`` = tokens / (forward + backward + optimizer) and
  ``model_duty_fraction`` (backend.rs:1807-1915). Multi-GPU figures take the max over
  ranks of each phase's time. On CUDA each phase is also an NVTX range, so a timeline
  profiler shows the phases.
* ``theoretical_forward_flops``: the reference's forward FLOP terms per step
  (burn_dragon_language/src/train/utils.rs:130-154: encoder, attention scores, attention
  values, decoder; backward about twice the forward), summed over the layers (its log
  line counts one layer's worth), plus the terms it leaves out (the y projection and the
  output head) under separate keys.
"""

from __future__ import annotations

import json
import os
import time
from collections import defaultdict

import torch
import torch.distributed as dist


def profiling_enabled() -> bool:
    return os.environ.get("DragonModel_STAGE_PROFILE", "0") not in ("", "0", "false")


class StageProfiler:
    def __init__(self, device: torch.device | None = None, enabled: bool | None = None):
        self.enabled = profiling_enabled() if enabled is None else enabled
        self.cuda = device is not None and device.type == "cuda"
        self.device = device
        self.ms: dict[str, float] = defaultdict(float)
        self.calls: dict[str, int] = defaultdict(int)
        self._open: dict[str, object] = {}
        self.tokens = 0
        self._wall0 = time.perf_counter()
        self._pending: list[tuple[str, object, object]] = []
        self._nvtx: dict[str, int] = {}

    def start(self, phase: str) -> None:
        if not self.enabled:
            return
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._open[phase] = e
            self._nvtx[phase] = torch.cuda.nvtx.range_start(phase)
        else:
            self._open[phase] = time.perf_counter()

    def stop(self, phase: str) -> None:
        if not self.enabled or phase not in self._open:
            return
        s = self._open.pop(phase)
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._pending.append((phase, s, e))
            if phase in self._nvtx:
                torch.cuda.nvtx.range_end(self._nvtx.pop(phase))
        else:
            self.ms[phase] += (time.perf_counter() - s) * 1e3
        self.calls[phase] += 1

    def _drain(self) -> None:
        if self._pending:
            torch.cuda.synchronize(self.device)
            for phase, s, e in self._pending:
                self.ms[phase] += s.elapsed_time(e)
            self._pending = []

    def summary(self) -> dict:
        self._drain()
        ms = dict(self.ms)
        if dist.is_initialized() and self.cuda:
            keys = sorted(ms)
            t = torch.tensor([ms[k] for k in keys], device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = dict(zip(keys, t.tolist()))
        wall = time.perf_counter() - self._wall0
        model_ms = sum(v for k, v in ms.items() if k in ("forward_backward", "forward", "backward", "optimizer"))
        out = {"phases_ms": ms, "calls": dict(self.calls), "tokens": self.tokens,
               "wall_tokens_per_second": self.tokens / wall if wall > 0 else 0.0}
        if model_ms > 0:
            out["model_tokens_per_second"] = self.tokens / (model_ms / 1e3)
            out["model_duty_fraction"] = (model_ms / 1e3) / wall if wall > 0 else 0.0
        return out


def theoretical_forward_flops(cfg, batch: int, block: int) -> dict:
    """Forward FLOPs of one step of ``batch`` x ``block`` tokens."""
    bt = batch * block
    D, N, H, Nh, V = cfg.n_embd, cfg.latent_total, cfg.n_head, cfg.latent_per_head, cfg.vocab_size
    L = cfg.n_layer
    enc = 2 * bt * D * N * L
    scores = 2 * batch * H * block * block * Nh * L
    value = 2 * batch * H * block * block * D * L
    dec = 2 * bt * N * D * L
    out = {"encoder": enc, "attn_scores": scores, "attn_value": value, "decoder": dec,
           "total": enc + scores + value + dec}
    # not in the reference's estimate: the y projection (a @ encoder_v per head) and the head
    out["encoder_v"] = 2 * bt * H * D * Nh * L
    out["lm_head"] = 2 * bt * D * V
    out["total_with_y_and_head"] = out["total"] + out["encoder_v"] + out["lm_head"]
    return out


class MetricsLogger:
    def __init__(self, run_dir: str | None, rank: int = 0, every: int = 1, console: bool = True):
        self.rank = rank
        self.every = max(1, every)
        self.console = console and rank == 0
        self.fh = None
        if run_dir is not None and rank == 0:
            os.makedirs(os.path.join(run_dir, "events"), exist_ok=True)
            self.fh = open(os.path.join(run_dir, "events", "metrics.jsonl"), "a")

    def log(self, step: int, **kv) -> None:
        if step % self.every and not kv.get("force"):
            return
        kv.pop("force", None)
        rec = {"step": step, "time": time.time(), **{k: (float(v) if isinstance(v, torch.Tensor) else v)
                                                     for k, v in kv.items()}}
        if self.fh is not None:
            self.fh.write(json.dumps(rec) + "\n")
            self.fh.flush()
        if self.console:
            body = " ".join(f"{k}={v:.5g}" if isinstance(v, float) else f"{k}={v}" for k, v in rec.items()
                            if k not in ("time",))
            print(f"[train] {body}", flush=True)

    def close(self) -> None:
        if self.fh is not None:
            self.fh.close()
            self.fh = None

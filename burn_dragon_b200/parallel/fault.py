"""Failure detection for multi-process training, entirely on the host.

* ``Heartbeat``: every rank publishes a timestamp under ``bdh/hb/<rank>`` in the process
  group's key-value store from a daemon thread; ``check()`` (called between steps, before
  the next launch) raises ``PeerFailure`` when a peer's heartbeat is older than the
  timeout or a peer announced that it is leaving (``announce_exit``). A rank that dies or
  hangs is therefore noticed by the others at a step boundary instead of inside a
  collective.
* ``NonFiniteGuard``: stops training on a NaN / Inf loss, like the reference's
  interrupter (burn_dragon_language/src/train/schedule.rs:51-60).

The reference has no elastic DDP (a rank failure ends the run, which then resumes from
its last checkpoint); the same holds here: ``PeerFailure`` ends the step loop and
``train.loop`` resumes from the newest checkpoint on the next launch.
"""

from __future__ import annotations

import math
import threading
import time

import torch
import torch.distributed as dist


class PeerFailure(RuntimeError):
    pass


class NonFiniteLoss(RuntimeError):
    pass


def _store():
    from torch.distributed import distributed_c10d as c10d

    return c10d._get_default_store()


class Heartbeat:
    def __init__(self, interval: float = 0.5, timeout: float = 10.0, store=None, rank: int | None = None,
                 world: int | None = None, prefix: str = "bdh/hb"):
        self.store = store if store is not None else _store()
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._stop = threading.Event()
        self._beat()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def _beat(self) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", repr(time.time()))

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:
                return

    def announce_exit(self, reason: str = "exit") -> None:
        """Tell the peers that this rank leaves (between steps, nothing in flight)."""
        self.store.set(f"{self.prefix}/{self.rank}/left", reason)
        self.stop()

    def stop(self) -> None:
        self._stop.set()

    def check(self) -> None:
        now = time.time()
        for r in range(self.world):
            if r == self.rank:
                continue
            key = f"{self.prefix}/{r}"
            if self.store.check([f"{key}/left"]):
                raise PeerFailure(f"rank {r} left: {self.store.get(f'{key}/left').decode()}")
            if not self.store.check([key]):
                raise PeerFailure(f"rank {r} never published a heartbeat")
            age = now - float(self.store.get(key).decode())
            if age > self.timeout:
                raise PeerFailure(f"rank {r} heartbeat is {age:.1f}s old (timeout {self.timeout}s)")

    def wait_for_peers(self, timeout: float | None = None) -> None:
        """Block until every peer has published one heartbeat (start-up)."""
        deadline = time.time() + (timeout or self.timeout)
        keys = [f"{self.prefix}/{r}" for r in range(self.world)]
        while not self.store.check(keys):
            if time.time() > deadline:
                raise PeerFailure("peers did not start within the timeout")
            time.sleep(0.05)


class NonFiniteGuard:
    """Checks the loss every ``every`` steps (one host read) and raises on NaN / Inf."""

    def __init__(self, every: int = 1):
        self.every = max(1, every)

    def check(self, step: int, loss: torch.Tensor | float) -> None:
        if step % self.every:
            return
        v = float(loss)
        if not math.isfinite(v):
            raise NonFiniteLoss(f"non-finite train loss {v} at step {step}")

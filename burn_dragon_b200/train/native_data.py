"""Python face of the native batch loader (``csrc/host/loader.cpp``).

Worker threads fill a ring of host buffers (pinned when CUDA is present) with the
batches of upcoming steps; ``next()`` hands out the next step's ``(x, y)`` as views of
its buffer. A buffer goes back to the workers at the following ``next()`` — after the
CUDA event recorded by ``mark_consumed()`` (call it once the step has enqueued its
host-to-device copies) has completed, so an asynchronous copy never reads a buffer that
is being refilled.
"""

from __future__ import annotations

import os

import torch

_MOD = None


def _load():
    global _MOD
    if _MOD is None:
        from torch.utils.cpp_extension import load

        here = os.path.join(os.path.dirname(os.path.dirname(__file__)), "csrc", "host")
        build = os.path.join(here, "build")
        os.makedirs(build, exist_ok=True)
        _MOD = load(name="_bdh_host", sources=[os.path.join(here, "loader.cpp")], build_directory=build,
                    extra_cflags=["-O3", "-std=c++17"], verbose=False)
    return _MOD


class NativeBytes:
    def __init__(self, mode: str, batch: int, block: int, *, path: str = "", vocab: int = 256, seed: int = 1337,
                 rank: int = 0, world: int = 1, split: str = "train", ratio: float = 0.9, chunk: int = 0,
                 depth: int = 4, workers: int = 2, start_step: int = 0, pin: bool | None = None,
                 token_bytes: int = 1):
        """``token_bytes``: 1 for byte files, 2 for uint16 token files (BPE vocabularies)."""
        mod = _load()
        if mode == "stream" and chunk <= 0:
            raise ValueError("stream mode needs chunk > 0")
        width = (chunk if mode == "stream" else block) + 1
        pin = torch.cuda.is_available() if pin is None else pin
        self.bufs = [torch.empty(batch, width, dtype=torch.int64, pin_memory=pin) for _ in range(max(2, depth))]
        self.width = width
        self._l = mod.Loader(mode, path, batch, width - 1, vocab, seed, rank, world, ratio, split == "valid",
                             chunk, self.bufs, workers, start_step, token_bytes)
        self.mode = mode
        self._held: int | None = None
        self._event = None
        self.step = start_step

    def next(self):
        """(x, y[, reset]) of the next step; ``reset`` (stream mode) marks stream starts."""
        if self._held is not None:
            if self._event is not None:
                self._event.synchronize()
            self._l.release(self._held)
        slot, step = self._l.take()
        self._held, self._event = slot, None
        self.step = step + 1
        w = self.bufs[slot]
        x, y = w[:, :-1], w[:, 1:]
        if self.mode == "stream":
            per = max(1, (self._l.split_len() // w.shape[0] - 1) // (self.width - 1))
            return x, y, step % per == 0
        return x, y

    def mark_consumed(self) -> None:
        """Record that the current batch's copies are enqueued on the current CUDA stream."""
        if torch.cuda.is_available():
            self._event = torch.cuda.Event()
            self._event.record()

    def close(self) -> None:
        self._l.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

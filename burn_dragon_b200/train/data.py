"""Seeded synthetic byte-token data (uniform random bytes) and stream windows.

The random loader draws [B, T+1] windows of uniform bytes from a counter-seeded
generator, so every rank / step gets a distinct, reproducible batch (rank-sharded like
the reference's process-group data shard, burn_dragon_language/src/train/schedule.rs:
10249-10297). The streaming loader walks consecutive windows of fixed per-stream byte
sequences (the stateful-TBPTT batching of burn_dragon_language/src/dataset/scheduler.rs)
and reports which streams start a new document so the carried state can be reset.
"""

from __future__ import annotations

import torch


class RandomBytes:
    def __init__(self, batch: int, block: int, vocab: int = 256, seed: int = 1337, rank: int = 0,
                 world: int = 1, pin: bool = False):
        self.batch, self.block, self.vocab = batch, block, vocab
        self.seed, self.rank, self.world = seed, rank, world
        self.pin = pin
        self.step = 0

    def next(self) -> tuple[torch.Tensor, torch.Tensor]:
        g = torch.Generator()
        g.manual_seed(self.seed * 1_000_003 + self.step * self.world + self.rank)
        self.step += 1
        w = torch.randint(0, self.vocab, (self.batch, self.block + 1), generator=g, dtype=torch.int64)
        x, y = w[:, :-1].contiguous(), w[:, 1:].contiguous()
        if self.pin:
            x, y = x.pin_memory(), y.pin_memory()
        return x, y


class StreamingBytes:
    """Consecutive chunks of `streams` independent byte streams of length `stream_len`."""

    def __init__(self, streams: int, stream_len: int, chunk: int, vocab: int = 256, seed: int = 1337,
                 rank: int = 0):
        g = torch.Generator()
        g.manual_seed(seed * 7919 + rank)
        self.data = torch.randint(0, vocab, (streams, stream_len + 1), generator=g, dtype=torch.int64)
        self.chunk = chunk
        self.stream_len = stream_len
        self.pos = 0

    def next(self) -> tuple[torch.Tensor, torch.Tensor, bool]:
        """Returns (inputs, targets, reset) where reset marks the start of new documents."""
        reset = self.pos == 0
        s = self.pos
        x = self.data[:, s:s + self.chunk]
        y = self.data[:, s + 1:s + self.chunk + 1]
        self.pos += self.chunk
        if self.pos + self.chunk > self.stream_len:
            self.pos = 0
        return x.contiguous(), y.contiguous(), reset


class FileBytes:
    """Random [B, T+1] windows of a token file (memory-mapped; uint8 bytes, or uint16 ids
    when ``token_bytes`` = 2), split into train / valid by ``train_split_ratio`` (the
    reference's file-backed corpora, dataset/mod.rs)."""

    def __init__(self, path: str, batch: int, block: int, split: str = "train", ratio: float = 0.9,
                 seed: int = 1337, rank: int = 0, world: int = 1, token_bytes: int | None = None):
        import numpy as np

        if token_bytes is None:
            from .datasets import token_bytes as tb

            token_bytes = tb(path)
        data = np.memmap(path, dtype=np.uint8 if token_bytes == 1 else np.dtype("<u2"), mode="r")
        cut = int(len(data) * ratio)
        self.data = data[:cut] if split == "train" else data[cut:]
        if len(self.data) <= block + 1:
            raise ValueError(f"{path}: {split} split has only {len(self.data)} tokens for block {block}")
        self.batch, self.block = batch, block
        self.seed, self.rank, self.world = seed, rank, world
        self.step = 0

    def next(self) -> tuple[torch.Tensor, torch.Tensor]:
        import numpy as np

        g = np.random.default_rng(self.seed * 1_000_003 + self.step * self.world + self.rank)
        self.step += 1
        starts = g.integers(0, len(self.data) - self.block - 1, size=self.batch)
        w = np.stack([np.asarray(self.data[s:s + self.block + 1], dtype=np.int64) for s in starts])
        t = torch.from_numpy(w)
        return t[:, :-1].contiguous(), t[:, 1:].contiguous()

"""Native prefetching batch loader: determinism, file windows, streams (CPU)."""

import numpy as np
import torch

from burn_dragon_b200.train.native_data import NativeBytes, _load


def test_random_batches_are_a_function_of_step_and_rank():
    a = NativeBytes("random", 4, 16, seed=3, rank=1, world=2, workers=3, depth=5)
    first = [tuple(t.clone() for t in a.next()) for _ in range(6)]
    a.close()
    b = NativeBytes("random", 4, 16, seed=3, rank=1, world=2, workers=1, depth=2, start_step=2)
    again = [tuple(t.clone() for t in b.next()) for _ in range(4)]
    b.close()
    for (x1, y1), (x2, y2) in zip(first[2:], again):
        assert torch.equal(x1, x2) and torch.equal(y1, y2)
    x, y = first[0]
    assert x.shape == (4, 16) and torch.equal(x[:, 1:], y[:, :-1])
    assert not torch.equal(first[0][0], first[1][0])
    c = NativeBytes("random", 4, 16, seed=3, rank=0, world=2, workers=1)
    assert not torch.equal(c.next()[0], first[0][0])
    c.close()
    # roughly uniform over the vocabulary
    d = NativeBytes("random", 64, 511, seed=1, vocab=256)
    v = torch.cat([d.next()[0].reshape(-1) for _ in range(4)])
    d.close()
    counts = torch.bincount(v, minlength=256).float()
    assert float(counts.std() / counts.mean()) < 0.1


def test_file_windows_come_from_the_split(tmp_path):
    data = (np.arange(5000) % 251).astype(np.uint8)
    p = tmp_path / "d.bin"
    data.tofile(p)
    ld = NativeBytes("file", 8, 32, path=str(p), ratio=0.8, workers=2)
    for _ in range(3):
        x, y = ld.next()
        for row_x, row_y in zip(x, y):
            start = int(row_x[0])
            # consecutive bytes of the file (values count up mod 251)
            assert torch.equal(row_x, (torch.arange(32) + start) % 251)
            assert torch.equal(row_y, (torch.arange(32) + start + 1) % 251)
    ld.close()
    vd = NativeBytes("file", 2, 32, path=str(p), ratio=0.8, split="valid")
    assert vd._l.split_len() == 1000
    vd.close()


def test_stream_chunks_are_consecutive_and_flag_resets(tmp_path):
    data = np.arange(4 * 100, dtype=np.int64).astype(np.uint8)
    p = tmp_path / "s.bin"
    data.tofile(p)
    ld = NativeBytes("stream", 4, 0, path=str(p), ratio=1.0, chunk=24)
    seen = [ld.next() for _ in range(5)]
    ld.close()
    (x0, _, r0), (x1, _, r1) = seen[0], seen[1]
    assert r0 and not r1
    assert torch.equal(x1[:, 0], x0[:, 0] + 24 if x0.max() < 200 else x1[:, 0])
    assert int(x0[1, 0]) == 100  # stream 1 starts at byte 100
    assert seen[4][2]  # 4 whole chunks of 24 (+1) per 100-byte stream: wraps


def test_module_builds_without_cuda():
    assert _load().draw(1, 2, 3, 4) >= 0

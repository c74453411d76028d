"""Startup batch-size selection from the exact fused-workspace footprint (CPU)."""

import pytest

from burn_dragon_b200.config import AutoBatchSizeConfig, DragonConfig
from burn_dragon_b200.train.autotune import choose_batch_size, state_bytes, workspace_bytes


def test_workspace_bytes_scale_with_batch():
    c = DragonConfig.bdh_gpu()
    w1, w2 = workspace_bytes(c, 8, 512), workspace_bytes(c, 16, 512)
    assert 1.9 < w2 / w1 < 2.1
    # BDH-GPU at batch 32 x 512 holds ~22 GiB of activations
    assert 18 * 2**30 < workspace_bytes(c, 32, 512) < 26 * 2**30
    assert state_bytes(c) > 25_000_000 * 18


def test_choose_batch_size_binary_search_and_accumulation():
    c = DragonConfig.bdh_gpu()
    ab = AutoBatchSizeConfig(enabled=True, target_device_memory_mb=40 * 1024, max_batch_size=256)
    r = choose_batch_size(c, 512, ab, target_effective_batch=200)
    m = ab.probe_safety_margin
    assert (state_bytes(c) + workspace_bytes(c, r.batch_size, 512)) * m <= r.budget_bytes
    assert (state_bytes(c) + workspace_bytes(c, r.batch_size + 1, 512)) * m > r.budget_bytes
    assert r.gradient_accumulation_steps == -(-200 // r.batch_size)
    lin = choose_batch_size(c, 512, AutoBatchSizeConfig(enabled=True, target_device_memory_mb=40 * 1024,
                                                        max_batch_size=256, binary_search=False))
    assert lin.batch_size == r.batch_size
    with pytest.raises(ValueError):
        choose_batch_size(c, 512, AutoBatchSizeConfig(enabled=True, target_device_memory_mb=64))

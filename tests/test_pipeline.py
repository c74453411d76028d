"""Pipeline planner (CPU) and a 2-stage pipeline over gloo ranks whose summed stage
gradients equal the single-process gradients (mirrors the reference's
pipeline_stage_surrogate_backward_matches_full_pipeline_gradients,
burn_dragon_language/src/train/schedule.rs:17053)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.parallel.pipeline import partition, plan


def _check(p):
    C = p.stages * p.virtual
    for r, evs in enumerate(p.events):
        seen_f = set()
        for kind, mb, c in evs:
            assert c % p.stages == r
            if kind == "F":
                seen_f.add((mb, c))
            else:
                assert (mb, c) in seen_f
        assert len(evs) == 2 * p.micro * len([c for c in range(C) if c % p.stages == r])


@pytest.mark.parametrize("kind", ["gpipe", "1f1b", "interleaved"])
def test_plans_are_complete_and_ordered(kind):
    p = plan(8, 4, 8, kind, virtual=2)
    _check(p)
    assert 0.0 <= p.bubble < 1.0


def test_partition_and_bubbles():
    assert partition(6, 4) == [(0, 2), (2, 4), (4, 5), (5, 6)]
    g = plan(8, 4, 8, "gpipe")
    o = plan(8, 4, 8, "1f1b")
    assert abs(g.bubble - 3 / 11) < 0.05  # (P-1)/(m+P-1)
    assert max(o.peak_inflight) <= 4 and max(g.peak_inflight) == 8
    assert o.peak_inflight == [4, 3, 2, 1]
    i = plan(8, 4, 8, "interleaved", virtual=2)
    assert i.bubble <= o.bubble + 1e-9


def _cfg():
    return DragonConfig(n_layer=4, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                        rotary_embedding="rope")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, kind, x, y, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.parallel.pipeline import PipelineRunner

    model = BDH(_cfg(), seed=9)
    runner = PipelineRunner(model, plan(4, world, 4, kind), rank, x.shape[0] // 4, x.shape[1])
    loss = runner.step(x, y)
    out[rank] = (model.store.grad.clone(), None if loss is None else float(loss))
    dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["gpipe", "1f1b"])
def test_two_stage_pipeline_matches_full_model(kind):
    torch.manual_seed(1)
    x = torch.randint(0, 256, (8, 12))
    y = torch.randint(0, 256, (8, 12))
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _port(), kind, x, y, out), nprocs=2, join=True)
    from burn_dragon_b200.models.bdh import BDH

    ref = BDH(_cfg(), seed=9)
    loss = ref.loss(x, y)
    grads = torch.autograd.grad(loss, list(ref.parameters()), allow_unused=True)
    flat = torch.zeros_like(ref.store.grad)
    for p, g in zip(ref.parameters(), grads):
        if g is not None:
            p.grad.copy_(g)
    flat.copy_(ref.store.grad)
    assert torch.allclose(out[0][0], out[1][0])
    assert torch.allclose(out[0][0], flat, atol=1e-6, rtol=1e-4)
    assert abs(out[1][1] - float(loss)) < 1e-5


def test_pipeline_settings_take_the_reference_keys():
    from burn_dragon_b200.train.loop import _pipeline_settings

    assert _pipeline_settings({"microbatches": 8, "schedule": "interleaved_1f1b", "virtual_stages_per_rank": 2,
                               "stage_count": 4}, 4) == (8, "interleaved", 2)
    assert _pipeline_settings({"micro_batches": 6, "schedule": "gpipe"}, 2) == (6, "gpipe", 1)
    with pytest.raises(ValueError, match="stage_count"):
        _pipeline_settings({"stage_count": 2}, 4)

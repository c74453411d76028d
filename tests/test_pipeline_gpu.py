"""Two fused pipeline stages on 2 GPUs vs the single-GPU fused step (summed grads)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _cfg():
    from burn_dragon_b200.config import DragonConfig

    return DragonConfig(n_layer=4, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                        rotary_embedding="rope", init_std=0.1)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.parallel.pipeline import PipelineRunner, plan

    dev = torch.device("cuda", rank)
    model = BDH(_cfg(), device=dev, seed=9)
    g = torch.Generator().manual_seed(0)
    x = torch.randint(0, 256, (4, 128), generator=g).to(dev)
    y = torch.randint(0, 256, (4, 128), generator=g).to(dev)
    runner = PipelineRunner(model, plan(4, world, 2, "1f1b"), rank, 2, 128)
    loss = runner.step(x, y)
    torch.cuda.synchronize()
    grads = model.store.grad.clone()
    ref = BDH(_cfg(), device=dev, seed=9)
    ref_loss = (ref.fused_step(x[:2], y[:2], loss_scale=0.5) + ref.fused_step(x[2:], y[2:], accumulate=True,
                                                                              loss_scale=0.5)).item()
    rel = ((grads - ref.store.grad).norm() / ref.store.grad.norm()).item()
    out[rank] = (rel, None if loss is None else loss.item(), ref_loss)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_pipeline_matches_single_gpu():
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _port(), out), nprocs=2, join=True)
    for r in (0, 1):
        assert out[r][0] < 1e-3, out[r]
    assert abs(out[1][1] - out[1][2]) < 1e-4 * abs(out[1][2])

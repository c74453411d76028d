"""Data parallelism on CPU ranks (gloo): replicas stay identical and equal the
single-process step on the concatenated batch (mirrors the reference's local-DDP and
single-rank collective tests, burn_dragon_language/src/train/schedule.rs:16532,16784)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from burn_dragon_b200.config import DragonConfig


def _cfg():
    return DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                        rotary_embedding="rope")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, x, y, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from burn_dragon_b200.train.trainer import Trainer

    tr = Trainer(_cfg(), "cpu", lr=1e-2, seed=5)
    b = x.shape[0] // world
    for _ in range(2):
        tr.step(x[rank * b:(rank + 1) * b], y[rank * b:(rank + 1) * b])
    out[rank] = tr.model.store.data.clone()
    dist.destroy_process_group()


def test_two_rank_ddp_matches_single_process():
    torch.manual_seed(0)
    x = torch.randint(0, 256, (4, 8))
    y = torch.randint(0, 256, (4, 8))
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(2, _free_port(), x, y, out), nprocs=2, join=True)
    from burn_dragon_b200.train.trainer import Trainer

    single = Trainer(_cfg(), "cpu", lr=1e-2, seed=5)
    for _ in range(2):
        single.step(x, y)
    assert torch.allclose(out[0], out[1])
    assert torch.allclose(out[0], single.model.store.data, atol=1e-6)

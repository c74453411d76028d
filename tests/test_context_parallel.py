"""Context parallelism (exact state prefix) on 2 gloo ranks == the unsplit sequence."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from burn_dragon_b200.config import DragonConfig


def _cfg(rot):
    return DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                        rotary_embedding=rot)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, rot, x, y, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.parallel.cp import cp_step_grads

    model = BDH(_cfg(rot), seed=4).double()
    Tc = x.shape[1] // world
    loss = cp_step_grads(model, x[:, rank * Tc:(rank + 1) * Tc], y[:, rank * Tc:(rank + 1) * Tc])
    out[rank] = (float(loss), model.store.grad.clone())
    dist.destroy_process_group()


@pytest.mark.parametrize("rot", ["rope", "alibi"])
def test_context_parallel_matches_full_sequence(rot):
    torch.manual_seed(0)
    x = torch.randint(0, 256, (2, 12))
    y = torch.randint(0, 256, (2, 12))
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _port(), rot, x, y, out), nprocs=2, join=True)
    from burn_dragon_b200.models.bdh import BDH

    ref = BDH(_cfg(rot), seed=4).double()
    loss = ref.loss(x, y)
    grads = torch.autograd.grad(loss, list(ref.parameters()), allow_unused=True)
    for p, g in zip(ref.parameters(), grads):
        p.grad.copy_(g if g is not None else torch.zeros_like(p))
    assert abs(out[0][0] - float(loss)) < 1e-5  # the CE runs in fp32
    assert torch.allclose(out[0][1], ref.store.grad, atol=1e-6)
    assert torch.allclose(out[1][1], ref.store.grad, atol=1e-6)

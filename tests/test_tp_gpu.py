"""Head-aligned tensor parallelism (2 GPUs) vs the unsharded fused step, and gradient
accumulation over micro-batches vs one batch (1 GPU)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _cfg():
    from burn_dragon_b200.config import DragonConfig

    return DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                        rotary_embedding="alibi", init_std=0.1)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out, fused="1"):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0", BDH_TP_FUSED="0" if fused == "0" else "1")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.parallel.tp import TensorParallel

    cfg = _cfg()
    dev = torch.device("cuda", rank)
    full = BDH(cfg, device=dev, seed=11)
    g = torch.Generator().manual_seed(0)
    x = torch.randint(0, 256, (2, 128), generator=g).to(dev)
    y = torch.randint(0, 256, (2, 128), generator=g).to(dev)
    loss_full = full.fused_step(x, y).item()
    gf = {k: v.clone() for k, v in full.grad_dict().items()}
    tp = TensorParallel(sequence_parallel=fused == "sp")
    local = BDH(tp.local_config(cfg), device=dev, seed=11)
    tp.shard_from_full(local, full.param_dict(), cfg)
    local.tp = tp
    loss_tp = local.fused_step(x, y).item()
    gl = local.grad_dict()
    hs = tp.head_slice(cfg)
    Nh = cfg.latent_per_head
    rel = lambda a, b: ((a - b).norm() / (b.norm() + 1e-12)).item()  # noqa: E731
    res = {
        "loss": (loss_full, loss_tp),
        "encoder": rel(gl["encoder"], gf["encoder"][hs]),
        "encoder_v": rel(gl["encoder_v"], gf["encoder_v"][hs]),
        "decoder": rel(gl["decoder"], gf["decoder"][hs.start * Nh:hs.stop * Nh]),
    }
    for n in ("embed", "lm_head", "norm_gamma", "norm_beta"):
        res[n] = rel(gl[n], gf[n])
    out[rank] = res
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused", ["1", "0", "sp"])
def test_tensor_parallel_matches_unsharded(fused):
    """fused = "1": decoder sums through the scattered GEMM + peer all-gather; "0": NCCL;
    "sp": sequence parallel (residual rows sharded, bf16 rows gathered, reduce-scatter of
    the residual gradient)."""
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _port(), out, fused), nprocs=2, join=True)
    for r in (0, 1):
        res = out[r]
        a, b = res.pop("loss")
        assert abs(a - b) < 1e-3 * abs(a)
        for k, v in res.items():
            assert v < 0.02, f"rank {r} {k}: {v:.3e}"


def test_micro_batch_accumulation_matches_full_batch():
    from burn_dragon_b200.models.bdh import BDH

    cfg = _cfg()
    m = BDH(cfg, device="cuda", seed=4)
    x = torch.randint(0, 256, (4, 128), device="cuda")
    y = torch.randint(0, 256, (4, 128), device="cuda")
    l_full = m.fused_step(x, y).item()
    g_full = {k: v.clone() for k, v in m.grad_dict().items()}
    l_acc = (m.fused_step(x[:2], y[:2], loss_scale=0.5) + m.fused_step(x[2:], y[2:], accumulate=True,
                                                                         loss_scale=0.5)).item()
    g = m.grad_dict()
    assert abs(l_full - l_acc) < 1e-4 * abs(l_full)
    for k in g:
        r = ((g[k] - g_full[k]).norm() / (g_full[k].norm() + 1e-12)).item()
        assert r < 1e-3, f"{k}: {r:.3e}"

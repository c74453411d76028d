"""DiLoCo outer step over gloo ranks; EGGROLL population estimator vs backprop."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from burn_dragon_b200.config import DragonConfig


def _cfg():
    return DragonConfig(n_layer=1, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                        rotary_embedding="rope", initialization="simple_normal", init_std=0.05)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from burn_dragon_b200.parallel.diloco import DiLoCo
    from burn_dragon_b200.train.trainer import Trainer

    tr = Trainer(_cfg(), "cpu", lr=1e-2, seed=2)
    tr.world = 1  # inner steps are local
    d = DiLoCo(tr.model.store, inner_steps=2, outer_lr=0.5, codec="fp16")
    start = tr.model.store.data.clone()
    g = torch.Generator().manual_seed(rank)
    locals_ = []
    for _ in range(2):
        x = torch.randint(0, 256, (2, 8), generator=g)
        tr.step(x, x.roll(1, 1))
        if d.inner == 1:
            pass
        locals_.append(tr.model.store.data.clone())
        d.after_inner_step()
    out[rank] = (start, locals_[-1], tr.model.store.data.clone())
    dist.destroy_process_group()


def test_diloco_outer_step_averages_pseudo_gradients():
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _port(), out), nprocs=2, join=True)
    s0, l0, g0 = out[0]
    _, l1, g1 = out[1]
    assert torch.equal(g0, g1)  # replicas agree after the outer step
    delta = ((s0 - l0).half().float() + (s0 - l1).half().float()) / 2
    want = s0 - 0.5 * (delta + 0.9 * delta)  # nesterov, first step
    assert torch.allclose(g0, want, atol=1e-5, rtol=1e-3)  # fp16 pseudo-gradient codec


def test_eggroll_estimate_correlates_with_gradient():
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.train.eggroll import es_gradient_estimate, es_step

    torch.manual_seed(0)
    model = BDH(_cfg(), seed=3)
    x = torch.randint(0, 256, (2, 8))
    y = torch.randint(0, 256, (2, 8))
    loss = model.loss(x, y)
    g = torch.autograd.grad(loss, [model.encoder])[0]
    est = es_gradient_estimate(model, x, y, population=512, sigma=1e-3, rank=4)["encoder"]
    cos = torch.nn.functional.cosine_similarity(est.flatten(), -g.flatten(), dim=0)
    assert cos > 0.12, float(cos)  # random directions would give ~0.001
    before = float(model.loss(x, y))
    for i in range(5):
        es_step(model, x, y, population=64, sigma=1e-3, lr=0.5, rank=4, seed=i)
    assert float(model.loss(x, y)) < before


def test_hybrid_layout():
    from burn_dragon_b200.parallel.tp import hybrid_layout

    tp, dp = hybrid_layout(8, 4)
    assert tp == [[0, 1, 2, 3], [4, 5, 6, 7]] and dp == [[0, 4], [1, 5], [2, 6], [3, 7]]


def test_eggroll_chunking_and_decay_match_one_batch():
    import copy

    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.train.eggroll import es_step

    cfg = DragonConfig(n_layer=1, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, vocab_size=32, dropout=0.0)
    m1 = BDH(cfg, seed=2)
    m2 = copy.deepcopy(m1)
    x = torch.randint(0, 32, (2, 8))
    es_step(m1, x, x, population=4, sigma=0.05, lr=0.1, rank=2, seed=9, weight_decay=0.1)
    es_step(m2, x, x, population=4, sigma=0.05, lr=0.1, rank=2, seed=9, weight_decay=0.1, chunk=1)
    for n in ("encoder", "encoder_v", "decoder"):
        torch.testing.assert_close(getattr(m1, n), getattr(m2, n), atol=1e-6, rtol=1e-5)


def test_training_loop_with_the_eggroll_optimizer(tmp_path, monkeypatch, capsys):
    import json

    from burn_dragon_b200.cli.train import main

    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    main(["--config", cfg, "--set", "training.max_iters=2", "--set", 'optimizer.name="eggroll"',
          "--set", "optimizer.eggroll={sigma=0.02, fitness_normalization=\"rank\", coefficient_clip=10.0, "
                   "update={max_delta_rms=0.1}, population={population_size=4, population_chunk_size=1, rank=2}}",
          "--run-name", "egg"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None
    assert json.load(open(os.path.join(res["run_dir"], "run_info.json")))["training_path"] == "eggroll"

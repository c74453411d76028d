"""Local predictive coding: activity inference, layer-local derivatives (CPU)."""


import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.train.predictive_coding import LocalPredictiveCodingConfig, PCInferenceConfig, local_pc_step


def model():
    cfg = DragonConfig(n_layer=3, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope", initialization="simple_normal", vocab_size=32)
    return BDH(cfg, seed=0)


def batch(seed=0, B=2, T=6):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 32, (B, T), generator=g), torch.randint(0, 32, (B, T), generator=g)


def test_fixed_prediction_equals_backprop():
    m = model()
    x, y = batch()
    loss, rep = local_pc_step(m, x, y, LocalPredictiveCodingConfig(solver="fixed_prediction"))
    got = m.store.grad.clone()
    m.zero_grad(set_to_none=False)
    ref_loss = m.loss(x, y)
    ref = torch.autograd.grad(ref_loss, list(m.parameters()), allow_unused=True)
    flat = torch.zeros_like(got)
    for (n, p), g in zip(m.named_parameters(), ref):
        if g is not None:
            m.store.view(flat, n).copy_(g)
    torch.testing.assert_close(got, flat, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(loss, ref_loss.detach())


def test_zero_inference_steps_gives_only_head_and_local_terms():
    m = model()
    x, y = batch(1)
    cfg = LocalPredictiveCodingConfig(inference=PCInferenceConfig(steps=0))
    local_pc_step(m, x, y, cfg)
    g = m.grad_dict()
    # predictions equal the activities: every layer factor has zero error
    assert float(g["encoder"].abs().max()) < 1e-6 and float(g["decoder"].abs().max()) < 1e-6
    assert float(g["lm_head"].abs().sum()) > 0


def test_inference_descends_energy_for_both_solvers():
    for solver in ("synchronous_equilibrium", "reverse_gauss_seidel"):
        m = model()
        x, y = batch(2)
        cfg = LocalPredictiveCodingConfig(solver=solver, sync_diagnostics=True,
                                          inference=PCInferenceConfig(steps=4, step_size=0.05))
        _, rep = local_pc_step(m, x, y, cfg)
        assert rep.energy_after < rep.energy_before, (solver, rep)
        assert rep.global_backward_calls == 0 and rep.local_vjp_calls > 0
        assert float(m.grad_dict()["encoder"].abs().sum()) > 0


def test_derivatives_invariant_to_batch_duplication():
    m = model()
    x, y = batch(3)
    cfg = LocalPredictiveCodingConfig(inference=PCInferenceConfig(steps=3))
    local_pc_step(m, x, y, cfg)
    g1 = m.store.grad.clone()
    m2 = model()
    local_pc_step(m2, torch.cat([x, x]), torch.cat([y, y]), cfg)
    torch.testing.assert_close(m2.store.grad, g1, rtol=1e-4, atol=1e-7)


def test_gradient_fidelity_report():
    from burn_dragon_b200.cli.pc_gradient_fidelity import main as fidelity

    small = ["--n-layer", "2", "--n-embd", "16", "--n-head", "2", "--latent-total", "64", "--vocab-size", "32",
             "--batch-size", "2", "--block-size", "8"]
    out = fidelity(small + ["--solver", "fixed_prediction"])
    g = out["arms"][0]["report"]["global"]
    # fixed prediction chains the factor VJPs: exactly backpropagation
    assert abs(g["cosine"] - 1.0) < 1e-5 and g["relative_l2_error"] < 1e-4
    out = fidelity(small + ["--inference-steps", "1,2", "--step-sizes", "0.05"])
    assert len(out["arms"]) == 2
    for arm in out["arms"]:
        r = arm["report"]
        assert r["reference_backward_calls"] == 1 and -1.0 <= r["global"]["cosine"] <= 1.0
        assert {f["parameter_family"] for f in r["parameter_families"]} >= {"encoder", "decoder", "embed"}


def test_local_pc_runs_on_tbptt_streams(tmp_path, monkeypatch, capsys):
    import json
    import os

    from burn_dragon_b200.cli.train import main
    from burn_dragon_b200.train import predictive_coding as P

    calls = []
    real = P.local_pc_step

    def spy(model, x, y, cfg, mask=None, rho0s=None):
        calls.append(rho0s is not None)
        return real(model, x, y, cfg, mask=mask, rho0s=rho0s)

    monkeypatch.setattr(P, "local_pc_step", spy)
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    main(["--config", cfg, "--set", "training.block_size=32", "--set", 'training.algorithm="predictive_coding"',
          "--set", "training.tbptt_chunk_size=16", "--set", "training.tbptt_persist_across_steps=true",
          "--set", "training.max_iters=3", "--run-name", "pcs"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None
    assert calls == [False, True, False]  # a new stream, its continuation, a new stream

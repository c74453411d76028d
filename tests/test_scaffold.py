"""Random scaffold: generator contract, function preservation, adapter-only grads, folding."""
import copy

import pytest
import torch

from burn_dragon_b200.config import DragonConfig, RandomScaffoldConfig
from burn_dragon_b200.models import scaffold as S
from burn_dragon_b200.models.bdh import BDH


def _cfg(**kw):
    rs = RandomScaffoldConfig(enabled=True, seed=20260729, rank=4, alpha=16.0, scaling="rank_stabilized",
                              trainable_gain=True, **kw)
    return DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                        rotary_embedding="rope", random_scaffold=rs)


def test_fnv1a64_known_vector():
    assert S.fnv1a64("") == 0xCBF29CE484222325
    assert S.fnv1a64("a") == 0xAF63DC4C8601EC8C


def test_generator_statistics_and_determinism():
    w = S.scaffold_tensor_cpu(1, "shared.encoder", (64, 1024), 0.02)
    assert abs(float(w.mean())) < 1e-3 and abs(float(w.std()) - 0.02) < 1e-3
    assert torch.equal(w, S.scaffold_tensor_cpu(1, "shared.encoder", (64, 1024), 0.02))
    assert not torch.equal(w, S.scaffold_tensor_cpu(2, "shared.encoder", (64, 1024), 0.02))
    r = S.scaffold_tensor_cpu(1, "shared.decoder", (100,), 0.5, "rademacher")
    assert set(r.unique().tolist()) == {-0.5, 0.5}


def test_zero_b_is_function_preserving():
    cfg = _cfg()
    model = BDH(cfg, seed=1)
    dense_cfg = copy.deepcopy(cfg)
    dense_cfg.random_scaffold.enabled = False
    dense = BDH(dense_cfg, seed=1)
    with torch.no_grad():
        for n in ("embed", "lm_head", "norm_gamma", "norm_beta"):
            getattr(dense, n).copy_(getattr(model, n))
        for n in ("encoder", "encoder_v", "decoder"):
            getattr(dense, n).copy_(model.scaffold_base(n))
    x = torch.randint(0, 256, (2, 9))
    assert torch.allclose(model(x), dense(x), atol=1e-6)


def test_backward_reaches_adapters_not_base():
    model = BDH(_cfg(), seed=1)
    with torch.no_grad():
        model.encoder_b.normal_(0, 0.1)
    loss = model.loss(torch.randint(0, 256, (2, 9)), torch.randint(0, 256, (2, 9)))
    names = [n for n, _ in model.named_parameters()]
    grads = torch.autograd.grad(loss, [p for _, p in model.named_parameters()], allow_unused=True)
    g = dict(zip(names, grads))
    assert "encoder" not in names and "encoder_a" in names
    assert g["encoder_b"].abs().sum() > 0 and g["encoder_a"].abs().sum() > 0 and g["encoder_gain"].abs() > 0


def test_fold_for_inference_preserves_logits():
    model = BDH(_cfg(), seed=2)
    with torch.no_grad():
        for n in ("encoder_b", "encoder_v_b", "decoder_b"):
            getattr(model, n).normal_(0, 0.05)
    dense = model.fold_scaffold_for_inference()
    x = torch.randint(0, 256, (2, 7))
    assert torch.allclose(model(x), dense(x), atol=1e-5)


def test_manifest_guard():
    cfg = _cfg()
    man = S.manifest(cfg)
    S.check_manifest(man, cfg)
    other = copy.deepcopy(cfg)
    other.random_scaffold.seed = 7
    with pytest.raises(ValueError):
        S.check_manifest(man, other)
    assert man["trainable_adapter_elements"] < man["full_projection_elements"]


@pytest.mark.gpu
def test_device_generator_matches_host_oracle():
    cfg = _cfg()
    model = BDH(cfg, device="cuda", seed=1)
    for n in ("encoder", "decoder"):
        dev = model.scaffold_base(n).cpu()
        host = S.scaffold_tensor_cpu(cfg.random_scaffold.seed, S.PATHS[n], S.base_shape(cfg, n), cfg.init_std)
        assert torch.allclose(dev, host, atol=1e-7, rtol=1e-5)


@pytest.mark.gpu
def test_fused_scaffold_step_matches_reference():
    from burn_dragon_b200.models import reference as R

    rs = RandomScaffoldConfig(enabled=True, seed=20260729, rank=16, alpha=16.0, scaling="rank_stabilized",
                              trainable_gain=True)
    cfg = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                       rotary_embedding="rope", random_scaffold=rs, init_std=0.1)
    model = BDH(cfg, device="cuda", seed=3)
    with torch.no_grad():
        for n in ("encoder_b", "encoder_v_b", "decoder_b"):
            getattr(model, n).normal_(0, 0.05)
    model.store.refresh_shadow()
    torch.manual_seed(0)
    x = torch.randint(0, 256, (2, 128), device="cuda")
    y = torch.randint(0, 256, (2, 128), device="cuda")
    ref = BDH(cfg, device="cuda", seed=3)
    with torch.no_grad():
        ref.store.data.copy_(model.store.data)
    pd = ref.param_dict()
    logits, _ = R.bdh_forward(x, pd, cfg)
    loss_ref = R.cross_entropy(logits, y)
    names = [n for n, _ in ref.named_parameters()]
    params = [p for _, p in ref.named_parameters()]
    effs = [pd["encoder"], pd["encoder_v"], pd["decoder"]]
    out = torch.autograd.grad(loss_ref, params + effs, allow_unused=True)
    grads = dict(zip(names, out[:len(params)]))
    d_eff = dict(zip(("encoder", "encoder_v", "decoder"), out[len(params):]))
    loss = model.fused_step(x, y)
    torch.cuda.synchronize()
    assert abs(loss.item() - loss_ref.item()) < 2e-2 * loss_ref.item()
    g = model.grad_dict()
    for n in ("encoder_a", "encoder_b", "decoder_a", "decoder_b", "encoder_v_b", "embed"):
        rel = ((g[n] - grads[n]).norm() / (grads[n].norm() + 1e-12)).item()
        assert rel < 0.1, f"{n}: {rel:.3e}"
    for n in ("encoder", "encoder_v", "decoder"):
        rel = ((model._geff[n] - d_eff[n]).norm() / d_eff[n].norm()).item()
        assert rel < 0.08, f"d{n}: {rel:.3e}"
        # the gain gradient is a cancelling sum: judge it against the scale of its terms
        base = model.scaffold_base(n)
        scale = (d_eff[n] * base).abs().sum().item()
        assert abs(g[f"{n}_gain"].item() - grads[f"{n}_gain"].item()) < 0.05 * scale


@pytest.mark.gpu
def test_gain_grad_kernel_matches_host_sum():
    from burn_dragon_b200 import _ext

    cfg = _cfg()
    model = BDH(cfg, device="cuda", seed=1)
    dW = torch.randn(S.base_shape(cfg, "encoder"), device="cuda")
    out = torch.zeros(1, device="cuda")
    _ext.load().scaffold_gain_grad(model.scaffold_keys["encoder"], cfg.init_std, 0, dW, out)
    ref = (dW.double() * model.scaffold_base("encoder").double()).sum().item()
    assert abs(out.item() - ref) < 1e-4 * (dW.abs() * model.scaffold_base("encoder").abs()).sum().item()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["encoder", "decoder"])
@pytest.mark.parametrize("cached", [False, True])
def test_adapter_grad_kernel_matches_torch_and_is_deterministic(name, cached):
    """One pass over dW gives dA = s dW B^T, dB = s A^T dW and the gain gradient
    sum(dW * W_seed) (regenerated or cached base) against fp64 PyTorch; two runs agree
    bitwise (fixed-slot partials, fixed-order sums)."""
    from burn_dragon_b200 import _ext

    rs = RandomScaffoldConfig(enabled=True, seed=20260729, rank=16, alpha=16.0, scaling="rank_stabilized",
                              trainable_gain=True)
    cfg = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                       rotary_embedding="rope", random_scaffold=rs)
    model = BDH(cfg, device="cuda", seed=1)
    mod = _ext.load()
    shp = S.base_shape(cfg, name)
    Hm, I, O = (shp[0], shp[1], shp[2]) if len(shp) == 3 else (1, shp[0], shp[1])
    r = cfg.random_scaffold.rank
    g = torch.Generator(device="cuda").manual_seed(4)
    dW = torch.randn(Hm, I, O, device="cuda", generator=g)
    A = torch.randn(Hm, I, r, device="cuda", generator=g)
    B = torch.randn(Hm, r, O, device="cuda", generator=g)
    base = model.scaffold_base(name).reshape(Hm, I, O)
    s = 0.25
    outs = []
    for _ in range(2):
        dA, dB, gain = torch.empty_like(A), torch.empty_like(B), torch.empty(1, device="cuda")
        work = torch.empty(mod.scaffold_adapter_work(Hm, I, O, r), device="cuda")
        mod.scaffold_adapter_grad(model.scaffold_keys[name], cfg.init_std, model.scaffold_dist, Hm, I, O, r,
                                  dW, A, B, base.contiguous() if cached else None, s, dA, dB, gain, work)
        outs.append((dA.clone(), dB.clone(), gain.clone()))
    torch.cuda.synchronize()
    d, a, b = dW.double(), A.double(), B.double()
    ref_a = s * d @ b.transpose(-1, -2)
    ref_b = s * a.transpose(-1, -2) @ d
    ref_g = (d * base.double()).sum()
    dA, dB, gain = outs[0]
    assert torch.allclose(dA.double(), ref_a, rtol=1e-4, atol=1e-3 * ref_a.abs().max().item())
    assert torch.allclose(dB.double(), ref_b, rtol=1e-4, atol=1e-3 * ref_b.abs().max().item())
    assert abs(gain.item() - ref_g.item()) < 1e-4 * (d.abs() * base.double().abs()).sum().item()
    for x, y in zip(outs[0], outs[1]):
        assert torch.equal(x, y)

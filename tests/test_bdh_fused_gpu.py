"""The fused sm_100a BDH step vs the PyTorch fp32 reference (loss and every gradient)."""
import pytest
import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models import reference as R
from burn_dragon_b200.models.bdh import BDH

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("rotary", ["rope", "alibi"])
def test_fused_step_matches_reference(rotary):
    # iid neurons: the x5 weights below on top of heavy-tailed neuron gains push a few
    # neurons far enough that bf16 activations alone move the encoder_v gradient ~9%
    cfg = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                       rotary_embedding=rotary, initialization="near_critical", residual_scaling="family_default",
                       neuron_gains="iid")
    model = BDH(cfg, device="cuda", seed=5)
    # larger weights than N(0, .02) so that every path carries signal in bf16
    with torch.no_grad():
        for n in ("encoder", "encoder_v", "decoder"):
            getattr(model, n).mul_(5.0)
    model.store.refresh_shadow()
    torch.manual_seed(0)
    B, T = 2, 256
    tokens = torch.randint(0, 256, (B, T), device="cuda")
    targets = torch.randint(0, 256, (B, T), device="cuda")

    # reference in fp32 on the bf16-rounded weights the kernels see
    ref_params = {}
    for n, p in model.param_dict().items():
        if p is None:
            ref_params[n] = None
            continue
        q = p.detach().clone()
        if n in ("encoder", "encoder_v", "decoder", "lm_head"):
            q = q.bfloat16().float()
        ref_params[n] = q.requires_grad_(True)
    logits, _ = R.bdh_forward(tokens, ref_params, cfg)
    ref_loss = R.cross_entropy(logits, targets)
    ref_loss.backward()

    loss = model.fused_step(tokens, targets)
    torch.cuda.synchronize()
    from burn_dragon_b200.ops.gemm import check_errors

    check_errors(torch.device("cuda"))
    assert abs(loss.item() - ref_loss.item()) < 2e-2 * abs(ref_loss.item())
    grads = model.grad_dict()
    for n in ("lm_head", "decoder", "encoder_v", "encoder", "embed", "norm_gamma", "norm_beta"):
        r = _rel(grads[n], ref_params[n].grad)
        assert r < 0.08, f"{n}: rel err {r:.3e}"


@pytest.mark.parametrize("rotary", ["rope", "alibi"])
def test_fused_stateful_chunks_match_reference(rotary):
    """Stateful TBPTT: chunk 2 continues chunk 1's detached state (loss, grads, state)."""
    from burn_dragon_b200.models.state import ModelState

    cfg = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                       rotary_embedding=rotary)
    model = BDH(cfg, device="cuda", seed=7)
    with torch.no_grad():
        for n in ("encoder", "encoder_v", "decoder"):
            getattr(model, n).mul_(5.0)
    model.store.refresh_shadow()
    torch.manual_seed(1)
    B, T = 2, 128
    toks = torch.randint(0, 256, (B, 2 * T), device="cuda")
    tgts = torch.randint(0, 256, (B, 2 * T), device="cuda")

    ref_params = {}
    for n, p in model.param_dict().items():
        q = p.detach().clone()
        if n in ("encoder", "encoder_v", "decoder", "lm_head"):
            q = q.bfloat16().float()
        ref_params[n] = q.requires_grad_(True)
    with torch.no_grad():
        _, rhos1 = R.bdh_forward(toks[:, :T], ref_params, cfg, need_state=True)
    logits2, rhos2 = R.bdh_forward(toks[:, T:], ref_params, cfg, rho0s=[r.detach() for r in rhos1], pos0=T,
                                   need_state=True)
    ref_loss = R.cross_entropy(logits2, tgts[:, T:])
    ref_loss.backward()

    st = ModelState.empty()
    model.fused_step(toks[:, :T], tgts[:, :T], state=st)
    for r_ref, r_got in zip(rhos1, st.rhos):
        assert _rel(r_got, r_ref) < 0.03
    loss = model.fused_step(toks[:, T:], tgts[:, T:], state=st)
    torch.cuda.synchronize()
    assert st.position == 2 * T
    assert abs(loss.item() - ref_loss.item()) < 2e-2 * abs(ref_loss.item())
    grads = model.grad_dict()
    for n in ("lm_head", "decoder", "encoder_v", "encoder", "embed"):
        r = _rel(grads[n], ref_params[n].grad)
        assert r < 0.08, f"{n}: rel err {r:.3e}"
    for r_ref, r_got in zip(rhos2, st.rhos):
        assert _rel(r_got, r_ref.detach()) < 0.03


def test_fused_step_at_bench_shape_default_init():
    """The BDH-GPU layer shape the benchmark runs (d=256, h=4, Nh=8192, T=512; B=2, L=2)
    with the default initialisation (heavy-tailed neuron gains), against the fp32
    PyTorch oracle on the same bf16-rounded weights. Exercises K = 8192 reductions, the
    CTA-pair kernels and the 256 x 256 TMA-epilogue tiles."""
    cfg = DragonConfig.bdh_gpu()
    cfg.n_layer = 2
    model = BDH(cfg, device="cuda", seed=11)
    torch.manual_seed(2)
    B, T = 2, 512
    tokens = torch.randint(0, 256, (B, T), device="cuda")
    targets = torch.randint(0, 256, (B, T), device="cuda")
    ref_params = {}
    for n, p in model.param_dict().items():
        if p is None:
            ref_params[n] = None
            continue
        q = p.detach().clone()
        if n in ("encoder", "encoder_v", "decoder", "lm_head"):
            q = q.bfloat16().float()
        ref_params[n] = q.requires_grad_(True)
    logits, _ = R.bdh_forward(tokens, ref_params, cfg)
    ref_loss = R.cross_entropy(logits, targets)
    ref_loss.backward()
    loss = model.fused_step(tokens, targets)
    torch.cuda.synchronize()
    from burn_dragon_b200.ops.gemm import check_errors

    check_errors(torch.device("cuda"))
    assert abs(loss.item() - ref_loss.item()) < 1e-2 * abs(ref_loss.item())
    grads = model.grad_dict()
    errs = {n: _rel(grads[n], ref_params[n].grad) for n in
            ("lm_head", "decoder", "encoder_v", "encoder", "embed", "norm_gamma", "norm_beta")}
    print("bench-shape relative gradient errors:", {k: f"{v:.3e}" for k, v in errs.items()})
    for n, r in errs.items():
        assert r < 0.08, f"{n}: rel err {r:.3e}"


def test_fused_step_is_bitwise_reproducible():
    """Race check: the fused step (split-K decoder partials in fixed slots, weight-gradient
    accumulation in stream order, row-kernel partials in fixed slots, no atomics) gives
    bitwise identical loss and gradients when run twice on the same inputs."""
    cfg = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                       rotary_embedding="rope")
    model = BDH(cfg, device="cuda", seed=21)
    torch.manual_seed(3)
    x = torch.randint(0, 256, (4, 256), device="cuda")
    y = torch.randint(0, 256, (4, 256), device="cuda")
    l1 = model.fused_step(x, y).clone()
    g1 = model.store.grad.clone()
    l2 = model.fused_step(x, y).clone()
    torch.cuda.synchronize()
    assert torch.equal(l1, l2)
    assert torch.equal(g1, model.store.grad)


@pytest.mark.parametrize("V,D,R", [(256, 256, 4096), (3000, 96, 1000)])
def test_embed_grad_kernel_matches_index_add(V, D, R):
    """The embedding-gradient kernel (scan form for small vocabularies, stable-sort form
    for large ones) against an fp32 index_add_, and bitwise equal across two calls."""
    from burn_dragon_b200 import _ext
    from burn_dragon_b200.models.bdh_fused import embed_grad

    mod = _ext.load()
    g = torch.Generator(device="cuda").manual_seed(5)
    tok = torch.randint(0, V, (R,), device="cuda", generator=g)
    rows = torch.randn(R, D, device="cuda", generator=g)
    base = torch.randn(V, D, device="cuda", generator=g)
    ref = base.double().index_add_(0, tok, rows.double()).float()
    out1 = base.clone()
    embed_grad(mod, tok, rows, out1, accumulate=True)
    out2 = base.clone()
    embed_grad(mod, tok, rows, out2, accumulate=True)
    fresh = torch.full_like(base, 7.0)
    embed_grad(mod, tok, rows, fresh, accumulate=False)
    torch.cuda.synchronize()
    assert torch.allclose(out1, ref, rtol=1e-5, atol=1e-4)
    assert torch.equal(out1, out2)
    assert torch.allclose(fresh, ref - base, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("kind", ["rms_norm", "dynamic_tanh", "derf"])
def test_fused_step_norm_kinds_match_reference(kind):
    """RMSNorm / DynamicTanh / Derf in the row kernels (embedding norm, attention-output
    norm, both residual-merge norms) against the fp32 PyTorch oracle, including the
    gradients of the learnable alpha / shift scalars."""
    cfg = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                       rotary_embedding="rope", initialization="near_critical", residual_scaling="family_default",
                       neuron_gains="iid", norm_kind=kind, norm_shift_init=0.1 if kind == "derf" else 0.0)
    model = BDH(cfg, device="cuda", seed=11)
    assert model._fused is None
    with torch.no_grad():
        for n in ("encoder", "encoder_v", "decoder"):
            getattr(model, n).mul_(5.0)
    model.store.refresh_shadow()
    torch.manual_seed(2)
    B, T = 2, 256
    tokens = torch.randint(0, 256, (B, T), device="cuda")
    targets = torch.randint(0, 256, (B, T), device="cuda")
    ref_params = {}
    for n, p in model.param_dict().items():
        if p is None:
            ref_params[n] = None
            continue
        q = p.detach().clone()
        if n in ("encoder", "encoder_v", "decoder", "lm_head"):
            q = q.bfloat16().float()
        ref_params[n] = q.requires_grad_(True)
    logits, _ = R.bdh_forward(tokens, ref_params, cfg)
    ref_loss = R.cross_entropy(logits, targets)
    ref_loss.backward()

    loss = model.fused_step(tokens, targets)
    torch.cuda.synchronize()
    from burn_dragon_b200.ops.gemm import check_errors

    check_errors(torch.device("cuda"))
    assert abs(loss.item() - ref_loss.item()) < 2e-2 * abs(ref_loss.item())
    grads = model.grad_dict()
    names = ["lm_head", "decoder", "encoder_v", "encoder", "embed", "norm_gamma", "norm_beta"]
    if kind != "rms_norm":
        names.append("norm_alpha")
    if kind == "derf":
        names.append("norm_shift")
    for n in names:
        r = _rel(grads[n], ref_params[n].grad)
        assert r < 0.08, f"{kind} {n}: rel err {r:.3e}"

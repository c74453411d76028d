"""fp64 gradient checks of the reference math (CPU): the analytic dense-attention
backward the fused kernels implement against autograd, and gradcheck of one BDH layer."""

import pytest
import torch

from burn_dragon_b200.models import reference as R


@pytest.mark.parametrize("decay", [False, True])
@pytest.mark.parametrize("with_state", [False, True])
def test_dense_attention_vjp_matches_autograd(decay, with_state):
    torch.manual_seed(0)
    B, H, T, N, D = 2, 3, 7, 5, 4
    dt = torch.float64
    q = torch.randn(B, H, T, N, dtype=dt, requires_grad=True)
    v = torch.randn(B, 1, T, D, dtype=dt, requires_grad=True)
    rho0 = torch.randn(B, H, N, D, dtype=dt, requires_grad=True) if with_state else None
    g = R.decay_vector([0.1, 0.3, 0.7], dtype=dt) if decay else None
    c, rho = R.linear_attention_dense(q, v, rho0=rho0, decay=g, need_state=True)
    dc, drho = torch.randn_like(c), torch.randn_like(rho)
    ins = [q, v] + ([rho0] if with_state else [])
    auto = torch.autograd.grad((c * dc).sum() + (rho * drho).sum(), ins)
    dq, dv, drho0 = R.linear_attention_dense_vjp(q.detach(), v.detach(), dc, rho0=None if rho0 is None else
                                                 rho0.detach(), decay=g, drho=drho)
    torch.testing.assert_close(dq, auto[0])
    torch.testing.assert_close(dv, auto[1])
    if with_state:
        torch.testing.assert_close(drho0, auto[2])


def test_bdh_layer_gradcheck():
    torch.manual_seed(1)
    dt = torch.float64
    B, T, D, H, Nh = 1, 4, 4, 2, 4
    v = torch.randn(B, T, D, dtype=dt, requires_grad=True)
    enc = (0.5 * torch.randn(H, D, Nh, dtype=dt)).requires_grad_(True)
    enc_v = (0.5 * torch.randn(H, D, Nh, dtype=dt)).requires_grad_(True)
    dec = (0.5 * torch.randn(H * Nh, D, dtype=dt)).requires_grad_(True)
    gamma = torch.ones(D, dtype=dt, requires_grad=True)
    beta = torch.zeros(D, dtype=dt, requires_grad=True)
    freqs = R.rope_freqs(Nh, 10000.0, dtype=dt)
    pos = torch.arange(T)

    def f(v, enc, enc_v, dec, gamma, beta):
        # a negative threshold keeps the ReLUs away from their kink at these sizes
        return R.bdh_layer(v, enc, enc_v, dec, gamma, beta, eps=1e-5, thr=-0.05, freqs=freqs, positions=pos,
                           decay=None)[0]

    assert torch.autograd.gradcheck(f, (v, enc, enc_v, dec, gamma, beta), eps=1e-6, atol=1e-5)


@pytest.mark.parametrize("decay", [False, True])
@pytest.mark.parametrize("T,chunk", [(40, 16), (48, 16), (33, 7)])
def test_row_chunked_attention_matches_dense(decay, T, chunk):
    """Row-chunked dense scores with the state carried between chunks: same output, final
    state and gradients (through the carried states) as the full dense form, in fp64."""
    from burn_dragon_b200.models import reference as R

    g = torch.Generator().manual_seed(T + chunk)
    B, H, N, D = 2, 3, 8, 5
    q = torch.randn(B, H, T, N, generator=g, dtype=torch.float64, requires_grad=True)
    v = torch.randn(B, 1, T, D, generator=g, dtype=torch.float64, requires_grad=True)
    rho0 = torch.randn(B, H, N, D, generator=g, dtype=torch.float64, requires_grad=True)
    dec = torch.tensor([0.9, 0.97, 0.8], dtype=torch.float64) if decay else None
    a1, r1 = R.linear_attention_dense(q, v, rho0=rho0, decay=dec)
    a2, r2 = R.linear_attention_chunked(q, v, rho0=rho0, decay=dec, chunk=chunk)
    assert torch.allclose(a1, a2, atol=1e-10) and torch.allclose(r1, r2, atol=1e-10)
    w1, w2 = torch.randn_like(a1), torch.randn_like(r1)
    g1 = torch.autograd.grad((a1 * w1).sum() + (r1 * w2).sum(), (q, v, rho0))
    g2 = torch.autograd.grad((a2 * w1).sum() + (r2 * w2).sum(), (q, v, rho0))
    for x, y in zip(g1, g2):
        assert torch.allclose(x, y, atol=1e-9)

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

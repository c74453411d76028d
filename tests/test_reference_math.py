"""CPU oracle contracts (mirrors the reference's model-math tests)."""
import math

import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models import reference as R
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.models.state import ModelState


def test_recurrent_equals_dense_score_without_decay():
    torch.manual_seed(0)
    q = torch.randn(2, 3, 17, 8, dtype=torch.float64)
    v = torch.randn(2, 1, 17, 5, dtype=torch.float64)
    rho0 = torch.randn(2, 3, 8, 5, dtype=torch.float64)
    c1, r1 = R.linear_attention_recurrent(q, v, rho0)
    c2, r2 = R.linear_attention_dense(q, v, rho0)
    assert torch.allclose(c1, c2, atol=1e-10)
    assert torch.allclose(r1, r2, atol=1e-10)


def test_recurrent_equals_dense_score_with_decay():
    torch.manual_seed(1)
    q = torch.randn(2, 3, 13, 8, dtype=torch.float64)
    v = torch.randn(2, 1, 13, 5, dtype=torch.float64)
    rho0 = torch.randn(2, 3, 8, 5, dtype=torch.float64)
    decay = R.decay_vector([1.0, 0.5, 0.25], dtype=torch.float64)
    c1, r1 = R.linear_attention_recurrent(q, v, rho0, decay)
    c2, r2 = R.linear_attention_dense(q, v, rho0, decay)
    assert torch.allclose(c1, c2, atol=1e-10)
    assert torch.allclose(r1, r2, atol=1e-10)


def test_attention_is_strictly_causal():
    q = torch.randn(1, 1, 6, 4, dtype=torch.float64)
    v = torch.randn(1, 1, 6, 3, dtype=torch.float64)
    c, _ = R.linear_attention_dense(q, v)
    assert torch.all(c[:, :, 0] == 0)  # first token sees an empty state
    v2 = v.clone()
    v2[:, :, 3] += 1.0
    c2, _ = R.linear_attention_dense(q, v2)
    assert torch.allclose(c[:, :, :4], c2[:, :, :4])  # diagonal excluded


def test_rope_frequencies_and_rotation():
    f = R.rope_freqs(8, 65536.0, dtype=torch.float64)
    assert math.isclose(float(f[0]), 1.0 / (2 * math.pi), rel_tol=1e-6)
    assert float(f[0]) == float(f[1])
    x = torch.randn(3, 8, dtype=torch.float64)
    ph = R.rope_phases(torch.arange(3), f).double()
    y = R.rope_apply(x, ph)
    # rotation preserves each pair's norm
    assert torch.allclose(x.view(3, 4, 2).norm(dim=-1), y.view(3, 4, 2).norm(dim=-1))
    assert torch.allclose(y[0], x[0])


def test_rho_can_be_signed():
    q = torch.rand(1, 1, 4, 3, dtype=torch.float64)
    v = -torch.rand(1, 1, 4, 2, dtype=torch.float64)
    _, rho = R.linear_attention_dense(q, v)
    assert (rho < 0).all()


def test_incremental_forward_matches_full_sequence():
    cfg = DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope")
    model = BDH(cfg).double()
    tokens = torch.randint(0, 256, (2, 12))
    full = model(tokens)
    st = ModelState.empty()
    a = model(tokens[:, :5], state=st)
    b = model(tokens[:, 5:], state=st)
    assert torch.allclose(torch.cat([a, b], 1), full, atol=1e-9)


def test_incremental_matches_full_with_alibi():
    cfg = DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="alibi")
    model = BDH(cfg).double()
    tokens = torch.randint(0, 256, (1, 9))
    full = model(tokens)
    st = ModelState.empty()
    parts = [model(tokens[:, i:i + 3], state=st) for i in range(0, 9, 3)]
    assert torch.allclose(torch.cat(parts, 1), full, atol=1e-9)


def test_flat_decoder_equals_headwise_sum():
    torch.manual_seed(3)
    B, H, T, Nh, D = 2, 3, 5, 4, 6
    yn = torch.randn(B, H, T, Nh, dtype=torch.float64)
    dec = torch.randn(H * Nh, D, dtype=torch.float64)
    flat = yn.permute(0, 2, 1, 3).reshape(B, T, H * Nh) @ dec
    head = sum(yn[:, h] @ dec[h * Nh:(h + 1) * Nh] for h in range(H))
    assert torch.allclose(flat, head)

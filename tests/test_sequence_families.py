"""Gated DeltaNet-2 and Mamba-3 sequence memories (CPU oracles and runtime integration)."""

import math

import pytest
import torch

from burn_dragon_b200.config import DragonConfig, GatedDeltaNet2Config, MambaSequenceConfig
from burn_dragon_b200.models.dragon_runtime import DragonRuntime, RuntimeState
from burn_dragon_b200.models.sequence import GDN2Params, Mamba3Params, gdn2_chunk_wy, gdn2_recurrent


def t4(vals, shape):
    return torch.tensor(vals, dtype=torch.float64).reshape(shape)


def test_gdn2_one_step_update():
    q = t4([0.7, -0.3], (1, 1, 1, 2))
    k = t4([0.4, 0.6], (1, 1, 1, 2))
    v = t4([0.8, -0.5, 0.25], (1, 1, 1, 3))
    e = t4([0.25, 0.75], (1, 1, 1, 2))
    w = t4([0.5, 0.2, 0.9], (1, 1, 1, 3))
    g = t4([math.log(0.5), math.log(0.25)], (1, 1, 1, 2))
    S0 = t4([0.2, -0.1, 0.05, 0.3, 0.4, -0.2], (1, 1, 2, 3))
    out, S = gdn2_recurrent(q, k, v, e, w, g, S0)
    dec = S0[0, 0] * torch.tensor([[0.5], [0.25]], dtype=torch.float64)
    ek = torch.tensor([0.25 * 0.4, 0.75 * 0.6], dtype=torch.float64)
    u = w[0, 0, 0] * v[0, 0, 0] - ek @ dec
    S_exp = dec + torch.outer(k[0, 0, 0], u)
    torch.testing.assert_close(S[0, 0], S_exp)
    torch.testing.assert_close(out[0, 0, 0], (q[0, 0, 0] @ S_exp) / math.sqrt(2))


@pytest.mark.parametrize("chunk", [1, 3, 8, 64])
def test_gdn2_chunk_wy_matches_recurrence(chunk):
    g = torch.Generator().manual_seed(0)
    B, H, T, L, D = 2, 3, 13, 4, 5
    r = lambda *s: torch.rand(*s, generator=g, dtype=torch.float64)
    q, k = r(B, H, T, L) - 0.5, r(B, H, T, L) - 0.5
    v, w = r(B, 1, T, D), r(B, H, T, D)
    e = r(B, H, T, L)
    ld = -r(B, H, T, L) * 0.3
    S0 = r(B, H, L, D) - 0.5
    o1, s1 = gdn2_recurrent(q, k, v, e, w, ld, S0)
    o2, s2 = gdn2_chunk_wy(q, k, v, e, w, ld, S0, chunk)
    torch.testing.assert_close(o2, o1)
    torch.testing.assert_close(s2, s1)
    # continuity across a state hand-off
    oa, sa = gdn2_chunk_wy(q[:, :, :6], k[:, :, :6], v[:, :, :6], e[:, :, :6], w[:, :, :6], ld[:, :, :6], S0, chunk)
    ob, sb = gdn2_chunk_wy(q[:, :, 6:], k[:, :, 6:], v[:, :, 6:], e[:, :, 6:], w[:, :, 6:], ld[:, :, 6:], sa, chunk)
    torch.testing.assert_close(torch.cat([oa, ob], 2), o1)
    torch.testing.assert_close(sb, s1)


def test_gdn2_projections_gate_modes():
    g = torch.Generator().manual_seed(1)
    for mode in ("channel", "scalar", "disabled"):
        cfg = GatedDeltaNet2Config(erase_gate=mode, write_gate=mode, decay_gate=mode, allow_neg_eigval=True)
        p = GDN2Params(2, 8, 4, cfg, g)
        key, erase, write, ld = p.project(torch.randn(2, 5, 8, generator=g))
        assert key.shape == (2, 2, 5, 4) and write.shape == (2, 2, 5, 8)
        if mode == "disabled":
            assert float(erase.min()) == 1.0 and float(ld.abs().max()) == 0.0
        else:
            assert float(erase.max()) <= 2.0 and float(ld.max()) <= 0.0
        if mode == "scalar":
            assert torch.allclose(erase, erase[..., :1].expand_as(erase))


def test_mamba3_chunking_and_state_carry_are_consistent():
    torch.manual_seed(0)
    cfg = MambaSequenceConfig(d_state=8, headdim=8, expand=2, chunk_size=64)
    p = Mamba3Params(16, cfg, torch.Generator().manual_seed(2)).double()
    h = torch.randn(2, 11, 16, dtype=torch.float64)
    full, st = p(h, None)
    p.chunk = 1  # one token per chunk: the plain recurrence
    tok, st1 = p(h, None)
    torch.testing.assert_close(tok, full)
    for k in st:
        torch.testing.assert_close(st1[k], st[k])
    p.chunk = 4
    a, sa = p(h[:, :5], None)
    b, sb = p(h[:, 5:], sa)
    torch.testing.assert_close(torch.cat([a, b], 1), full)
    torch.testing.assert_close(sb["ssm"], st["ssm"])


def test_mamba3_gradients_finite():
    cfg = MambaSequenceConfig(d_state=8, headdim=8, expand=2, chunk_size=4)
    p = Mamba3Params(16, cfg, torch.Generator().manual_seed(3))
    out, _ = p(torch.randn(2, 9, 16), None)
    out.square().mean().backward()
    assert all(torch.isfinite(q.grad).all() for q in p.parameters())


def tiny(**kw):
    c = DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                     rotary_embedding="rope", initialization="simple_normal", vocab_size=64)
    for key, val in kw.items():
        setattr(c, key, val)
    return c


@pytest.mark.parametrize("fam,ex", [("gated_deltanet2", "reference"), ("gated_deltanet2", "gated_delta_chunk_wy"),
                                    ("mamba3_state_space_duality", "reference")])
def test_runtime_with_sequence_family_streams(fam, ex):
    cfg = tiny(sequence_memory_system=fam, sequence_executor=ex)
    cfg.mamba.headdim = 16
    cfg.mamba.chunk_size = 3
    cfg.gated_deltanet2.chunk_size = 3
    rt = DragonRuntime(cfg, seed=4)
    t = torch.randint(0, 64, (2, 7), generator=torch.Generator().manual_seed(5))
    full = rt.forward(t)
    st = RuntimeState.new(2)
    parts = [rt.forward(t[:, :4], st), rt.forward(t[:, 4:], st)]
    torch.testing.assert_close(torch.cat(parts, 1), full, rtol=1e-4, atol=1e-5)
    loss = rt.loss(t, t)
    loss.backward()
    assert torch.isfinite(loss)
    extra = rt.gdn2 if fam == "gated_deltanet2" else rt.mamba
    assert any(p.grad is not None and float(p.grad.abs().sum()) > 0 for p in extra.parameters())


def test_unsupported_family_executor_rejected():
    with pytest.raises(ValueError):
        tiny(sequence_memory_system="mamba3_state_space_duality", sequence_executor="gated_delta_chunk_wy").validate()


@pytest.mark.parametrize("T,chunk", [(11, 4), (16, 8), (7, 64)])
def test_mamba3_vectorised_path_matches_chunk_loop(T, chunk):
    """The whole-sequence preprocessing of the device path (with the PyTorch scan oracle)
    equals the chunk loop, outputs and carried state, including a carried-in state."""
    from burn_dragon_b200.models.sequence import ssd_scan_reference

    cfg = MambaSequenceConfig(d_state=8, headdim=8, expand=2, chunk_size=chunk)
    p = Mamba3Params(16, cfg, torch.Generator().manual_seed(5)).double()
    h = torch.randn(2, T, 16, dtype=torch.float64)
    _, st0 = p(torch.randn(2, 3, 16, dtype=torch.float64), None)
    ref, sr = p(h, st0)
    got, sg = p.forward_fused(h, st0, scan=ssd_scan_reference)
    torch.testing.assert_close(got, ref)
    for k in sr:
        torch.testing.assert_close(sg[k], sr[k])


@pytest.mark.gpu
@pytest.mark.parametrize("T,chunk,S,P", [(200, 64, 16, 128), (37, 8, 8, 32)])
def test_ssd_chunk_kernels_match_torch(T, chunk, S, P):
    """``ssd_chunk_fwd`` / ``ssd_chunk_bwd`` against the PyTorch scan (fp32 oracle, autograd
    for the backward): outputs, final state and every input gradient."""
    from burn_dragon_b200.models.sequence import SSDChunkScan, ssd_scan_reference

    g = torch.Generator(device="cuda").manual_seed(1)
    BH, n = 6, -(-T // chunk)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)  # noqa: E731
    da = -(torch.rand(BH, T, device="cuda", generator=g) * 0.1)
    da = torch.cat([c.cumsum(1) for c in da.split(chunk, 1)], 1)
    ins = [r(BH, T, S) * 0.5, r(BH, T, S) * 0.5, r(BH, T, P), da, r(BH, P, S) * 0.1, r(BH, n, P), r(BH, n, S),
           torch.rand(BH, n, device="cuda", generator=g)]
    a = [t.clone().requires_grad_(True) for t in ins]
    b = [t.clone().requires_grad_(True) for t in ins]
    y1, s1 = SSDChunkScan.apply(*a, chunk)
    y2, s2 = ssd_scan_reference(*b, chunk)
    torch.testing.assert_close(y1, y2, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(s1, s2, rtol=1e-4, atol=1e-4)
    wy, ws = r(BH, T, P), r(BH, P, S)
    ((y1 * wy).sum() + (s1 * ws).sum()).backward()
    ((y2 * wy).sum() + (s2 * ws).sum()).backward()
    for name, x1, x2 in zip(("q", "k", "v", "da", "s0", "vs", "ks", "cf"), a, b):
        err = (x1.grad - x2.grad).abs().max().item()
        scale = x2.grad.abs().max().item() + 1e-6
        assert err < 1e-3 * scale + 1e-4, f"d{name}: {err:.3e} (scale {scale:.3e})"


@pytest.mark.gpu
def test_mamba3_device_path_matches_chunk_loop():
    cfg = MambaSequenceConfig(d_state=16, headdim=32, expand=2, chunk_size=16)
    p = Mamba3Params(64, cfg, torch.Generator().manual_seed(7)).cuda()
    h = torch.randn(2, 70, 64, device="cuda")
    got, sg = p(h, None)  # CUDA: the ssd_chunk kernels
    from burn_dragon_b200.models.sequence import ssd_scan_reference

    ref, sr = p.forward_fused(h, None, scan=ssd_scan_reference)
    torch.testing.assert_close(got, ref, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(sg["ssm"], sr["ssm"], rtol=1e-3, atol=1e-3)

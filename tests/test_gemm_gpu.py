"""tcgen05 GEMM engine vs a plain PyTorch fp32 reference of the same op."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from burn_dragon_b200.ops import gemm as G

    return G


def _ref(a, b, a_t, b_t):
    A = a.float().t() if a_t else a.float()
    B = b.float().t() if b_t else b.float()
    return A @ B


def _close(got, ref, tol=2e-2):
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, f"max rel err {err / scale:.3e}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 128, 192), (384, 64, 1024), (200, 96, 136)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
def test_matmul_layouts(M, N, K, a_t, b_t):
    G = _ops()
    torch.manual_seed(0)
    dev = "cuda"
    a = torch.randn((K, M) if a_t else (M, K), device=dev).bfloat16()
    b = torch.randn((N, K) if b_t else (K, N), device=dev).bfloat16()
    got = G.matmul(a, b, a_t=a_t, b_t=b_t)
    torch.cuda.synchronize()
    G.check_errors(torch.device(dev))
    _close(got, _ref(a, b, a_t, b_t))


def test_split_k_partials_sum():
    G = _ops()
    torch.manual_seed(1)
    M, N, K, S = 256, 256, 2048, 4
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(K, N, device="cuda").bfloat16()
    out = torch.empty(S, M, N, device="cuda")
    G.gemm(G.EPI_F32, G.Operand(a, False, K, M, K), G.Operand(b, True, N, K, N), M, N, K, out, splits=S, ld=N,
           split_stride=M * N)
    torch.cuda.synchronize()
    _close(out.sum(0), _ref(a, b, False, False))


def test_batched_z_coordinates_and_accumulate():
    G = _ops()
    torch.manual_seed(2)
    Z, M, N, K = 3, 128, 128, 256
    a = torch.randn(Z, M, K, device="cuda").bfloat16()
    b = torch.randn(Z, N, K, device="cuda").bfloat16()
    out = torch.ones(Z, M, N, device="cuda")
    G.gemm(G.EPI_F32, G.Operand(a, False, K, M, K, z1=(Z, M * K)), G.Operand(b, False, K, N, K, z1=(Z, N * K)),
           M, N, K, out, Z1=Z, ld=N, sz1=M * N, accumulate=True)
    torch.cuda.synchronize()
    _close(out - 1.0, torch.bmm(a.float(), b.float().transpose(1, 2)))


def test_causal_scores_epilogue():
    G = _ops()
    torch.manual_seed(3)
    B, H, T, Nh = 2, 2, 256, 128
    q = torch.randn(B, T, H, Nh, device="cuda").bfloat16()
    S = torch.full((B, H, T, T), 7.0, device="cuda").bfloat16()
    op = G.Operand(q, False, Nh, T, H * Nh, z1=(H, Nh), z2=(B, T * H * Nh))
    G.gemm(G.EPI_SCORES, op, op, T, T, Nh, S, Z1=H, Z2=B, bn=128, causal_skip=True, ld=T, sz1=T * T,
           sz2=H * T * T)
    torch.cuda.synchronize()
    qf = q.float().permute(0, 2, 1, 3)
    ref = torch.tril(qf @ qf.transpose(-1, -2), diagonal=-1)
    _close(S, ref)
    assert (S.float().triu() == 0).all()


@pytest.mark.parametrize("a_t,b_t,N", [(True, False, 256), (False, False, 256), (False, True, 256),
                                       (False, True, 128)])
@pytest.mark.parametrize("M,K", [(256, 512), (640, 1024)])
def test_cta_pair_kernel_matches_single_cta(a_t, b_t, N, M, K):
    """The cta_group::2 kernel (256-row tiles on a CTA pair) equals the 1-CTA kernel."""
    G = _ops()
    torch.manual_seed(5)
    a = torch.randn((K, M) if a_t else (M, K), device="cuda").bfloat16()
    b = torch.randn((N, K) if b_t else (K, N), device="cuda").bfloat16()
    A = G.Operand(a, True, M, K, M) if a_t else G.Operand(a, False, K, M, K)
    B = G.Operand(b, False, K, N, K) if b_t else G.Operand(b, True, N, K, N)
    o1 = torch.empty(M, N, device="cuda")
    o2 = torch.empty(M, N, device="cuda")
    G.gemm(G.EPI_F32, A, B, M, N, K, o1, ld=N, pair=False)
    G.gemm(G.EPI_F32, A, B, M, N, K, o2, ld=N, pair=True)
    torch.cuda.synchronize()
    G.check_errors(torch.device("cuda"))
    assert torch.allclose(o1, o2, rtol=1e-5, atol=1e-3)
    _close(o2, _ref(a, b, a_t, b_t))


def test_cta_pair_causal_scores():
    G = _ops()
    torch.manual_seed(6)
    B, H, T, Nh = 2, 2, 512, 256
    q = torch.randn(B, T, H, Nh, device="cuda").bfloat16()
    op = G.Operand(q, False, Nh, T, H * Nh, z1=(H, Nh), z2=(B, T * H * Nh))
    outs = []
    for pair in (False, True):
        S = torch.full((B, H, T, T), 3.0, device="cuda").bfloat16()
        G.gemm(G.EPI_SCORES, op, op, T, T, Nh, S, Z1=H, Z2=B, bn=256, causal_skip=True, ld=T, sz1=T * T,
               sz2=H * T * T, pair=pair)
        outs.append(S)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def _tma_case(case, B=2, T=256, D=64, H=2, Nh=512, seed=0, table=False):
    """Operands of one TMA-epilogue BDH contraction (the layouts of the fused step) and a
    call that runs it with a given tile N; returns (call, outputs)."""
    G = _ops()
    Op = G.Operand
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: (torch.randn(*s, device="cuda", generator=g) * 0.5).bfloat16()  # noqa: E731
    N, M = H * Nh, B * T
    freq = torch.rand(Nh, device="cuda", generator=g) * 0.1
    tab = G.rope_table(freq, 0, T) if table else None
    if case == "xproj":
        v, enc = r(M, D), r(H, D, Nh)
        outs = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
        call = lambda bn: G.gemm(G.EPI_RELU_ROPE, Op(v, False, D, M, D), Op(enc, True, Nh, D, Nh, z1=(H, D * Nh)),  # noqa: E731
                                 M, Nh, D, outs[0], Z1=H, bn=bn, out1=outs[1], ld=N, sz1=Nh, thr=0.1, freq=freq, T=T,
                                 Nh=Nh, rope_tab=tab)
    elif case == "gate":
        an, encv, x = r(M, H, D), r(H, D, Nh), torch.relu(r(M, N).float()).bfloat16()
        outs = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16)]
        call = lambda bn: G.gemm(G.EPI_GATE, Op(an, False, D, M, H * D, z1=(H, D)),  # noqa: E731
                                 Op(encv, True, Nh, D, Nh, z1=(H, D * Nh)), M, Nh, D, outs[0], Z1=H, bn=bn, aux0=x,
                                 ld=N, sz1=Nh, thr=0.05)
    elif case == "dec_bwd":
        dm, dec = r(M, D), r(N, D)
        x = torch.relu(r(M, N).float()).bfloat16()
        yn = (torch.relu(r(M, N).float()) * x.float()).bfloat16()
        outs = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
        call = lambda bn: G.gemm(G.EPI_DEC_BWD, Op(dm, False, D, M, D), Op(dec, False, D, N, D), M, N, D,  # noqa: E731
                                 outs[0], bn=bn, out1=outs[1], aux0=x, aux1=yn, ld=N)
    else:  # dq: dx_part carries the x <= 0 mask as -0.0
        g16, q = r(B, H, T, T), r(M, N)
        dx0 = r(M, N)
        dx0 = torch.where(torch.rand(M, N, device="cuda", generator=g) < 0.3, torch.full_like(dx0, -0.0), dx0)
        outs = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16)]

        def call(bn):
            outs[0].copy_(dx0)
            G.gemm(G.EPI_DQ, Op(g16, False, T, T, T, z1=(H, T * T), z2=(B, H * T * T)),
                   Op(q, True, Nh, T, N, z1=(H, Nh), z2=(B, T * N)), T, Nh, T, outs[0], Z1=H, Z2=B, bn=bn,
                   aux0=outs[0], ld=N, sz1=Nh, sz2=T * N, freq=freq, T=T, Nh=Nh, rope_tab=tab)
    return call, outs


@pytest.mark.parametrize("case", ["xproj", "gate", "dec_bwd", "dq"])
def test_tma_epilogue_pair256_matches_single_cta128(case):
    """The CTA-pair 256 x 256 TMA-epilogue kernel (two 64-column chunks per epilogue warp)
    against the 1-CTA 128 x 128 kernel on the same operands: same per-element math, so
    the outputs agree to the bf16 rounding of the accumulator."""
    G = _ops()
    call, outs = _tma_case(case)
    call(128)
    ref = [o.float().clone() for o in outs]
    call(256)
    torch.cuda.synchronize()
    G.check_errors(torch.device("cuda"))
    for got, r in zip(outs, ref):
        _close(got, r, tol=1e-2)
        # the masked (-0.0) / zero pattern is identical
        assert torch.equal(got == 0, r == 0)


@pytest.mark.parametrize("case", ["xproj", "dq"])
def test_rope_table_matches_evaluated_phases(case):
    """The half2 (cos, sin) table path of the RoPE epilogues against the per-element
    evaluation of the same phases (fp16 phase values: agreement to the bf16 output)."""
    G = _ops()
    c0, o0 = _tma_case(case, table=False)
    c1, o1 = _tma_case(case, table=True)
    # the x-projection stages table tiles through its TMA ring (both tile widths); dQ
    # reads the table with plain loads
    for bn in (128, 256):
        c0(bn)
        c1(bn)
        torch.cuda.synchronize()
        G.check_errors(torch.device("cuda"))
        for a, b in zip(o0, o1):
            _close(b, a.float(), tol=1e-2)


@pytest.mark.parametrize("bn", [128, 256])
def test_decoder_backward_and_dq_epilogues_match_fp32(bn):
    """The decoder-backward epilogue (dx_part = g yn / x on x > 0, else the -0.0 mask
    marker; dy = g x on yn > 0) and the dQ epilogue (dx = dx_part + rope^T(G q) on live
    entries, the marker kept) against fp32 PyTorch on the same bf16 operands."""
    from burn_dragon_b200.models.reference import rope_freqs

    G = _ops()
    Op = G.Operand
    B, T, D, H, Nh = 2, 256, 64, 2, 512
    N, M = H * Nh, B * T
    g = torch.Generator(device="cuda").manual_seed(3)
    r = lambda *s: (torch.randn(*s, device="cuda", generator=g) * 0.5).bfloat16()  # noqa: E731
    dm, dec = r(M, D), r(N, D)
    x = torch.relu(r(M, N).float()).bfloat16()
    yn = (torch.relu(r(M, N).float()) * x.float()).bfloat16()
    dxp, dy = (torch.empty(M, N, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    G.gemm(G.EPI_DEC_BWD, Op(dm, False, D, M, D), Op(dec, False, D, N, D), M, N, D, dxp, bn=bn, out1=dy, aux0=x,
           aux1=yn, ld=N)
    acc = dm.float() @ dec.float().t()
    xf, yf = x.float(), yn.float()
    ref_dy = torch.where(yf > 0, acc * xf, torch.zeros_like(acc))
    ref_dxp = torch.where(xf > 0, acc * yf / xf.clamp_min(1e-30), torch.zeros_like(acc))
    torch.cuda.synchronize()
    G.check_errors(torch.device("cuda"))
    _close(dy, ref_dy, tol=1e-2)
    _close(dxp, ref_dxp, tol=1e-2)
    marker = dxp.view(torch.int16) == -32768  # bf16 -0.0
    assert torch.equal(marker, x.float() <= 0)

    # dQ over the decoder-backward output
    g16, q = r(B, H, T, T), r(M, N)
    freq = rope_freqs(Nh, 10000.0, device="cuda")
    dx = dxp.clone()
    G.gemm(G.EPI_DQ, Op(g16, False, T, T, T, z1=(H, T * T), z2=(B, H * T * T)),
           Op(q, True, Nh, T, N, z1=(H, Nh), z2=(B, T * N)), T, Nh, T, dx, Z1=H, Z2=B, bn=bn, aux0=dx, ld=N,
           sz1=Nh, sz2=T * N, freq=freq, T=T, Nh=Nh)
    gq = torch.einsum("bhts,bshj->bthj", g16.float(), q.float().view(B, T, H, Nh))  # [B, T, H, Nh]
    pos = torch.arange(T, device="cuda", dtype=torch.float32)
    raw = pos[:, None] * freq[0::2][None, :]
    ph = (raw - torch.round(raw)) * (2 * torch.pi)
    c, s = torch.cos(ph)[None, :, None, :], torch.sin(ph)[None, :, None, :]
    ge, go = gq[..., 0::2], gq[..., 1::2]
    rot = torch.stack((ge * c + go * s, go * c - ge * s), dim=-1).reshape(B, T, H, Nh).reshape(M, N)
    ref_dx = torch.where(marker, torch.zeros_like(rot), rot + dxp.float())
    torch.cuda.synchronize()
    G.check_errors(torch.device("cuda"))
    _close(dx, ref_dx, tol=1e-2)
    assert torch.equal(dx.view(torch.int16) == -32768, marker)

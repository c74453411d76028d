"""Generation: CPU recurrent decode == full forward; GPU prefill/decode kernels vs oracle."""
import pytest
import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models import reference as R
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.models.generate import Generator, sample_next
from burn_dragon_b200.models.state import ModelState


def _cfg(rotary="rope"):
    return DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=8, dropout=0.0,
                        rotary_embedding=rotary)


def test_cpu_decode_matches_teacher_forced_forward():
    model = BDH(_cfg(), seed=2).double()
    g = Generator(model)
    toks = torch.randint(0, 256, (2, 10))
    full = model(toks)
    logits, st = g.prefill(toks[:, :6])
    assert torch.allclose(logits, full[:, 5].float(), atol=1e-5)
    for i in range(6, 10):
        logits = g.decode_step(toks[:, i], st)
        assert torch.allclose(logits, full[:, i].float(), atol=1e-5)


def test_sampling_modes():
    logits = torch.tensor([[0.0, 5.0, 1.0, 2.0]])
    assert int(sample_next(logits)) == 1
    g = torch.Generator().manual_seed(0)
    draws = {int(sample_next(logits, 1.0, top_k=2, generator=g)) for _ in range(50)}
    assert draws <= {1, 3}


def test_generate_greedy_cpu_shape():
    model = BDH(_cfg(), seed=4)
    out = Generator(model).generate(torch.randint(0, 256, (3, 5)), 7, device_buffer_tokens=3)
    assert out.shape == (3, 7)


@pytest.mark.gpu
def test_rho_step_kernel_matches_recurrence():
    from burn_dragon_b200 import _ext

    torch.manual_seed(0)
    B, H, Nh, D = 3, 2, 256, 64
    rho = torch.randn(B, H, Nh, D, device="cuda")
    q = torch.rand(B, H * Nh, device="cuda").bfloat16()
    v = torch.randn(B, D, device="cuda")
    gamma = torch.tensor([0.9, 0.5], device="cuda")
    a = torch.zeros(B, H, D, device="cuda")
    qh = q.float().view(B, H, Nh)
    ref_a = torch.einsum("bhn,bhnd->bhd", qh, rho)
    ref_rho = (rho + qh[..., None] * v[:, None, None, :]) * gamma.view(1, H, 1, 1)
    _ext.load().rho_step(rho, q, H * Nh, v, gamma, a, B, H, Nh, D)
    torch.cuda.synchronize()
    assert torch.allclose(a, ref_a, rtol=1e-4, atol=1e-3)
    assert torch.allclose(rho, ref_rho, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("rotary", ["rope", "alibi"])
@pytest.mark.parametrize("state_dtype", ["fp32", "bf16"])
def test_gpu_prefill_and_decode_match_reference(rotary, state_dtype):
    """Prefill + decode against the fp32 teacher-forced oracle; with a bf16 decode state
    the bound is the same (the state is rounded once per update)."""
    cfg = _cfg(rotary)
    model = BDH(cfg, device="cuda", seed=6)
    with torch.no_grad():
        for n in ("encoder", "encoder_v", "decoder"):
            getattr(model, n).mul_(5.0)
    model.store.refresh_shadow()
    params = {n: (p.detach().bfloat16().float() if n in ("encoder", "encoder_v", "decoder", "lm_head") else p.detach())
              for n, p in model.param_dict().items()}
    torch.manual_seed(3)
    B, T = 2, 256
    toks = torch.randint(0, 256, (B, T + 4), device="cuda")
    full, _ = R.bdh_forward(toks, params, cfg)
    g = Generator(model, prefill_chunk=128, state_dtype=state_dtype)
    logits, st = g.prefill(toks[:, :T])

    def rel(a, b):
        return ((a - b).norm() / b.norm()).item()

    assert rel(logits, full[:, T - 1]) < 0.03
    for i in range(T, T + 4):
        logits = g.decode_step(toks[:, i], st)
        assert rel(logits, full[:, i]) < 0.03, i
    if state_dtype == "bf16":
        assert st.rhos[0].dtype == torch.bfloat16


def test_ragged_batch_matches_serial_greedy():
    import torch

    from burn_dragon_b200.config import DragonConfig
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.models.generate import Generator

    cfg = DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope", initialization="simple_normal", vocab_size=64)
    m = BDH(cfg, seed=0)
    g = Generator(m)
    prompts = [[1, 2, 3], [4, 5, 6, 7, 8, 9], [10], [11, 12]]
    budgets = [5, 3, 0, 7]
    out = g.generate_ragged(prompts, budgets, device_buffer_tokens=4, device="cpu")
    for p, b, o in zip(prompts, budgets, out):
        if b == 0:
            assert o == []
            continue
        ref = g.generate(torch.tensor([p]), b)[0].tolist()
        assert o == ref
    # a stop token ends a row early (and is kept)
    first = out[0][1]
    stopped = g.generate_ragged([prompts[0]], [5], stop_token=first, device="cpu")[0]
    assert stopped == out[0][:2]


def test_stream_chunks_and_sliding_window():
    import torch

    from burn_dragon_b200.config import DragonConfig
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.models.generate import Generator

    cfg = DragonConfig(n_layer=1, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope", initialization="simple_normal", vocab_size=64)
    g = Generator(BDH(cfg, seed=1))
    chunks = []
    full = g.generate_stream([1, 2, 3, 4, 5], 7, chunk_tokens=3, on_chunk=chunks.append, device="cpu")
    assert [len(c) for c in chunks] == [3, 3, 1] and full[5:] == sum(chunks, [])
    ref = g.generate(torch.tensor([[1, 2, 3, 4, 5]]), 7)[0].tolist()
    assert full[5:] == ref
    win = g.generate_stream([9, 9, 1, 2, 3, 4, 5], 7, sliding_window=5, device="cpu")
    assert win == full


@pytest.mark.gpu
def test_ragged_batch_on_cuda_matches_serial():
    import torch

    from burn_dragon_b200.config import DragonConfig
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.models.generate import Generator

    cfg = DragonConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=16, dropout=0.0,
                       rotary_embedding="rope", initialization="simple_normal", vocab_size=256)
    g = Generator(BDH(cfg, device="cuda", seed=0), prefill_chunk=128)
    gen = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 256, (n,), generator=gen).tolist() for n in (130, 256, 7)]
    out = g.generate_ragged(prompts, [6, 4, 9], device_buffer_tokens=4)
    for p, b, o in zip(prompts, [6, 4, 9], out):
        assert o == g.generate(torch.tensor([p], device="cuda"), b)[0].tolist()

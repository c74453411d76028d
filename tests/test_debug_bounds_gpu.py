"""DRAGON_DEBUG_BOUNDS: the row kernels check data-dependent indices (token ids, targets)
against the vocabulary, record a code in the device's error word and skip the access."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_out_of_vocab_ids_are_reported_not_read():
    from burn_dragon_b200 import _ext
    from burn_dragon_b200.ops import gemm as G

    dev = torch.device("cuda", 0)
    mod = _ext.load()
    G.set_debug_bounds(dev, True)
    try:
        V, D, R = 64, 32, 16
        table = torch.randn(V, D, device=dev)
        gam, bet = torch.ones(D, device=dev), torch.zeros(D, device=dev)
        y = torch.zeros(R, D, device=dev)
        mean, rstd = torch.empty(R, device=dev), torch.empty(R, device=dev)
        good = torch.randint(0, V, (R,), device=dev)
        mod.ln_fwd(table, good, R, D, gam, bet, 1e-5, y, None, mean, rstd)
        G.check_errors(dev)  # in range: no report
        ref = torch.nn.functional.layer_norm(table[good], (D,), gam, bet, 1e-5)
        assert torch.allclose(y, ref, atol=1e-5)
        bad = good.clone()
        bad[3] = V + 1000  # would read past the table
        y.zero_()
        mod.ln_fwd(table, bad, R, D, gam, bet, 1e-5, y, None, mean, rstd)
        with pytest.raises(IndexError, match="201"):
            G.check_errors(dev)
        assert torch.equal(y[3], torch.zeros(D, device=dev))  # the row was skipped
        # cross-entropy target and embedding-gradient token checks
        logits = torch.randn(R, V, device=dev)
        loss_rows, dl = torch.empty(R, device=dev), torch.empty(R, V, device=dev, dtype=torch.bfloat16)
        inv = torch.full((1,), 1.0 / R, device=dev)
        mod.cross_entropy(logits, bad, None, inv, R, V, loss_rows, dl)
        with pytest.raises(IndexError, match="202"):
            G.check_errors(dev)
        out = torch.zeros(V, D, device=dev)
        mod.embed_grad(torch.where(bad > V, -bad, bad), torch.randn(R, D, device=dev), R, D, out, False, None, None)
        with pytest.raises(IndexError, match="203"):
            G.check_errors(dev)
    finally:
        G.set_debug_bounds(dev, False)
    # checks off: the error word stays clear on good ids
    mod.ln_fwd(table, good, R, D, gam, bet, 1e-5, y, None, mean, rstd)
    G.check_errors(dev)

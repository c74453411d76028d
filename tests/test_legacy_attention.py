"""Block patterns, legacy row-normalised attention and its KV cache, latent block masks (CPU)."""

import torch

from burn_dragon_b200.config import DragonConfig, training_config_from_dict
from burn_dragon_b200.models import reference as R
from burn_dragon_b200.models.dragon_runtime import DragonRuntime
from burn_dragon_b200.models.legacy_attention import (AttentionCache, BlockPattern1d, BlockPattern2d,
                                                      forward_cached, row_normalized_attention)


def naive(q, v, slopes=None, allowed=None):
    B, H, T, _ = q.shape
    out = torch.zeros(B, H, T, v.shape[-1], dtype=q.dtype)
    for i in range(T):
        row = []
        for j in range(i):
            s = (q[:, :, i] * q[:, :, j]).sum(-1)
            if slopes is not None:
                s = s + slopes * (j - i)
            if allowed is not None and not allowed(i, j):
                s = s * 0
            row.append(s)
        if not row:
            continue
        S = torch.stack(row, -1)
        S = S / (S.abs().sum(-1, keepdim=True) + 1e-6)
        out[:, :, i] = torch.einsum("bhj,bhjd->bhd", S, v.expand(B, H, T, v.shape[-1])[:, :, :i])
    return out


def test_row_normalized_matches_naive_with_alibi_and_block_pattern():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 2, 9, 4, generator=g, dtype=torch.float64)
    v = torch.randn(2, 1, 9, 3, generator=g, dtype=torch.float64)
    slopes = torch.tensor([0.5, 0.25], dtype=torch.float64)
    torch.testing.assert_close(row_normalized_attention(q, v, "alibi", None, slopes), naive(q, v, slopes.view(1, 2)))
    pat = BlockPattern2d(3, {(0, 0), (1, 1), (2, 0), (2, 2)})
    got = row_normalized_attention(q, v, "alibi", None, None, pat)
    torch.testing.assert_close(got, naive(q, v, None, lambda i, j: pat.is_active(i // 3, j // 3)))
    dense = row_normalized_attention(q, v, "alibi", None, None, BlockPattern2d(3))
    torch.testing.assert_close(dense, row_normalized_attention(q, v, "alibi"))


def test_kv_cache_decode_matches_full_pass():
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 2, 7, 8, generator=g, dtype=torch.float64)
    v = torch.randn(1, 1, 7, 3, generator=g, dtype=torch.float64)
    freqs = R.rope_freqs(8, 100.0, dtype=torch.float64)
    slopes = torch.tensor([0.5, 0.7], dtype=torch.float64)
    full = row_normalized_attention(q, v, "rope", freqs, slopes)
    cache = AttentionCache()
    parts = [forward_cached(q[:, :, :3], v[:, :, :3], cache, "rope", freqs, slopes)]
    parts += [forward_cached(q[:, :, t:t + 1], v[:, :, t:t + 1], cache, "rope", freqs, slopes) for t in range(3, 7)]
    torch.testing.assert_close(torch.cat(parts, 2), full)
    assert len(cache) == 7


def test_block_pattern_1d_mask():
    m = BlockPattern1d(4, {0, 2}).mask(10)
    assert m.tolist() == [1, 1, 1, 1, 0, 0, 0, 0, 1, 1]
    assert BlockPattern1d(4).mask(5).sum() == 5


def test_latent_block_mask_equals_zeroed_columns():
    cfg = DragonConfig(n_layer=2, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                       rotary_embedding="rope", initialization="simple_normal", vocab_size=32,
                       latent_block_size=8, latent_active_blocks=[1, 3])
    rt = DragonRuntime(cfg, seed=0)
    t = torch.randint(0, 32, (2, 6))
    out = rt.forward(t)
    keep = rt._latent_mask.bool()
    with torch.no_grad():
        rt.core.encoder[:, :, ~keep] = 0
        rt.core.encoder_v[:, :, ~keep] = 0
    ref = rt.core.forward(t)
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    rt.loss(t, t).backward()
    assert float(rt.core.encoder.grad[:, :, ~keep].abs().sum()) == 0.0
    c = training_config_from_dict({"model": {"n_embd": 16, "fused_kernels": {"block_sparse": {
        "latent": {"block_size": 16, "active_blocks": [2, 0]}}}}}).model
    assert c.latent_active_blocks == [0, 2] and c.latent_block_size == 16 and c.uses_extended_runtime()

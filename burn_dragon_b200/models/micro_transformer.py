"""Small pre-norm transformer block (burn_dragon_core/src/model/micro_transformer.rs).

``x + proj(softmax(QK^T / sqrt(d_h)) V)`` over LayerNorm(x), then ``x + W2 gelu(W1
LayerNorm(x))``. Attention is either full (no mask) or group-causal: position i
attends to position j when ``j // group <= i // group`` (micro_transformer.rs:115-132).
The attention is ``torch.nn.functional.scaled_dot_product_attention``; the block is a
utility for auxiliary heads, not part of the BDH hot path.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn


class MicroTransformerBlock(nn.Module):
    def __init__(self, dim: int, heads: int, mlp_ratio: int = 4):
        super().__init__()
        self.heads = max(heads, 1)
        self.head_dim = max(dim // self.heads, 1)
        self.norm_attn = nn.LayerNorm(dim)
        self.qkv = nn.Linear(dim, 3 * dim)
        self.proj = nn.Linear(dim, dim)
        self.norm_mlp = nn.LayerNorm(dim)
        self.mlp_in = nn.Linear(dim, max(dim * mlp_ratio, 1))
        self.mlp_out = nn.Linear(max(dim * mlp_ratio, 1), dim)

    def _attention(self, x: torch.Tensor, group: int | None) -> torch.Tensor:
        B, T, D = x.shape
        q, k, v = self.qkv(x).split(D, -1)
        sh = lambda t: t.view(B, T, self.heads, self.head_dim).transpose(1, 2)
        mask = None
        if group is not None:
            gid = torch.arange(T, device=x.device) // max(group, 1)
            mask = gid[None, :] <= gid[:, None]
        scale = 1.0 / max(math.sqrt(self.head_dim), 1.0)
        o = F.scaled_dot_product_attention(sh(q), sh(k), sh(v), attn_mask=mask, scale=scale)
        return self.proj(o.transpose(1, 2).reshape(B, T, D))

    def forward(self, x: torch.Tensor, group_size: int | None = None) -> torch.Tensor:
        if x.numel() == 0:
            return x
        x = x + self._attention(self.norm_attn(x), group_size)
        return x + self.mlp_out(F.gelu(self.mlp_in(self.norm_mlp(x))))
